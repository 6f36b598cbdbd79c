// troncons_b200 — the C-ABI entry points (include/troncons_b200.h): argument checks with the
// reference's rules (trc-noyaux/src/lib.rs `Noyaux`, `Erreur::Usage`), then the launches.
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <string>

#include "../../include/troncons_b200.h"
#include "commun.cuh"
#include "mxfp4.cuh"
#include "noyaux.h"

namespace {

thread_local std::string g_erreur;

int usage(const char* fmt, ...) {
    char b[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(b, sizeof b, fmt, ap);
    va_end(ap);
    g_erreur = b;
    return TRC_ERR_USAGE;
}

int statut(cudaError_t e) {
    if (e == cudaSuccess) {
        g_erreur.clear();
        return TRC_OK;
    }
    g_erreur = std::string("CUDA: ") + cudaGetErrorString(e);
    return TRC_ERR_CUDA;
}

bool aligne(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// This library links its own (static) CUDA runtime: before launching on the caller's stream,
// make this runtime's current device the stream's device (the caller may have chosen it
// through another runtime instance, e.g. PyTorch's).
cudaError_t sur_le_device_du_flux(void* flux) {
    if (flux == nullptr) return cudaSuccess;
    // A stream under graph capture refuses the device query; launches into it are recorded on
    // the device it was captured on, which an earlier eager call on the stream aligned.
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(static_cast<cudaStream_t>(flux), &capture) == cudaSuccess &&
        capture != cudaStreamCaptureStatusNone)
        return cudaSuccess;
    int d = -1, cur = -1;
    cudaError_t e = cudaStreamGetDevice(static_cast<cudaStream_t>(flux), &d);
    if (e != cudaSuccess) return e;
    e = cudaGetDevice(&cur);
    if (e != cudaSuccess) return e;
    return cur == d ? cudaSuccess : cudaSetDevice(d);
}

#define SUR_LE_FLUX(f)                                        \
    do {                                                      \
        const cudaError_t e_ = sur_le_device_du_flux(f);      \
        if (e_ != cudaSuccess) return statut(e_);             \
    } while (0)

tb::Dims dims_de(const trc_dims_expert* d) {
    tb::Dims r;
    for (int j = 0; j < 3; ++j) {
        r.lignes[j] = d->lignes[j];
        r.colonnes[j] = d->colonnes[j];
    }
    return r;
}

// DimsExpert::verifier (abi.rs:98-108).
int verifier_dims(const trc_dims_expert* d) {
    if (d == nullptr) return usage("dims absent");
    for (int j = 0; j < 3; ++j) {
        const uint32_t r = d->lignes[j], c = d->colonnes[j];
        if (r == 0 || c == 0 || c % 32 != 0) return usage("matrix %d: shape %u x %u (columns must be a multiple of 32)", j, r, c);
        if (uint64_t(r) * (c / 32) * 16 > 0xFFFFFFFFull) return usage("matrix %d: more than 4 GiB of codes", j);
    }
    return TRC_OK;
}

}  // namespace

namespace tb {

cudaError_t assurer_smem(const void* noyau, int octets) {
    static std::mutex mu;
    static std::map<std::pair<const void*, int>, int> fait;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> g(mu);
    int& v = fait[{noyau, dev}];
    if (v >= octets) return cudaSuccess;
    e = cudaFuncSetAttribute(noyau, cudaFuncAttributeMaxDynamicSharedMemorySize, octets);
    if (e == cudaSuccess) v = octets;
    return e;
}

int erreur_usage(const char* message) { return usage("%s", message); }
int erreur_cuda(cudaError_t e) { return statut(e); }
cudaError_t aligner_device(void* flux) { return sur_le_device_du_flux(flux); }

}  // namespace tb

extern "C" {

const char* trc_derniere_erreur(void) { return g_erreur.c_str(); }

uint64_t trc_taille_emplacement(const trc_dims_expert* dims) {
    if (dims == nullptr) return 0;
    uint64_t s = 0;
    for (int j = 0; j < 3; ++j) s += tb::disposition_matrice(dims->lignes[j], dims->colonnes[j]).pas;
    return s;
}

int trc_decoder_expert(const void* partie, size_t partie_octets, void* emplacement, size_t emplacement_octets,
                       const uint32_t* luts, size_t luts_octets, const trc_dims_expert* dims, uint32_t* controle,
                       size_t controle_octets, void* flux) {
    if (int s = verifier_dims(dims)) return s;
    if (partie == nullptr || partie_octets < 64) return usage("part of %zu bytes (a 64-byte header at least)", partie_octets);
    if (!aligne(partie, 16)) return usage("part not aligned on 16");
    if (emplacement == nullptr || emplacement_octets < trc_taille_emplacement(dims))
        return usage("slot of %zu bytes, %llu needed", emplacement_octets, (unsigned long long)trc_taille_emplacement(dims));
    if (!aligne(emplacement, 256)) return usage("slot not aligned on 256");
    if (luts == nullptr || luts_octets < 3u * 4u * 4096u * 4u || !aligne(luts, 16)) return usage("LUTs of %zu bytes (196,608, 16-aligned)", luts_octets);
    if (controle == nullptr || controle_octets < 16 || !aligne(controle, 4)) return usage("control buffer under 16 bytes");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_decodage(nullptr, 1, partie, partie_octets, emplacement, luts, dims_de(dims), controle,
                                      static_cast<cudaStream_t>(flux)));
}

int trc_decoder_lot(const trc_desc_decodage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims,
                    void* flux) {
    if (int s = verifier_dims(dims)) return s;
    if (n == 0 || n > 65535) return usage("batch of %u experts", n);
    if (descs == nullptr || descs_octets < size_t(n) * sizeof(trc_desc_decodage) || !aligne(descs, 8))
        return usage("descriptors too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_decodage(reinterpret_cast<const tb::DescDecodage*>(descs), n, nullptr, 0, nullptr, nullptr,
                                      dims_de(dims), nullptr, static_cast<cudaStream_t>(flux)));
}

int trc_copier_brut(const void* partie, size_t partie_octets, void* emplacement, size_t emplacement_octets,
                    const trc_dims_expert* dims, uint32_t* controle, size_t controle_octets, void* flux) {
    if (int s = verifier_dims(dims)) return s;
    if (partie == nullptr || partie_octets < 64 || !aligne(partie, 16)) return usage("part too short or not 16-aligned");
    if (emplacement == nullptr || emplacement_octets < trc_taille_emplacement(dims) || !aligne(emplacement, 256))
        return usage("slot too short or not 256-aligned");
    if (controle == nullptr || controle_octets < 16 || !aligne(controle, 4)) return usage("control buffer under 16 bytes");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_copier_brut(partie, partie_octets, emplacement, dims_de(dims), controle,
                                         static_cast<cudaStream_t>(flux)));
}

int trc_gemv(const void* matrice, size_t matrice_octets, const float* x, size_t x_octets, float* y, size_t y_octets,
             uint32_t lignes, uint32_t colonnes, void* flux) {
    if (lignes == 0 || colonnes == 0 || colonnes % 32 != 0) return usage("shape %u x %u", lignes, colonnes);
    if (uint64_t(lignes) * (colonnes / 32) * 16 > 0xFFFFFFFFull) return usage("more than 4 GiB of codes");
    const uint64_t pas = tb::disposition_matrice(lignes, colonnes).pas;
    if (matrice == nullptr || matrice_octets < pas) return usage("matrix of %zu bytes, %llu needed", matrice_octets, (unsigned long long)pas);
    if (!aligne(matrice, 256)) return usage("matrix not aligned on 256");
    if (x == nullptr || x_octets < 4ull * colonnes || !aligne(x, 16)) return usage("x too short or not aligned on 16");
    if (y == nullptr || y_octets < 4ull * lignes) return usage("y too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_gemv(matrice, x, y, lignes, colonnes, static_cast<cudaStream_t>(flux)));
}

int trc_gemv_lot(const trc_desc_gemv* descs, size_t descs_octets, uint32_t n, uint32_t lignes_max, void* flux) {
    if (n == 0 || n > 65535) return usage("batch of %u products", n);
    if (descs == nullptr || descs_octets < size_t(n) * sizeof(trc_desc_gemv) || !aligne(descs, 8))
        return usage("descriptors too short");
    if (lignes_max == 0) return usage("lignes_max = 0");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_gemv_lot(reinterpret_cast<const tb::DescGemv*>(descs), n, lignes_max,
                                      static_cast<cudaStream_t>(flux)));
}

int trc_gemv_f32(const float* w, size_t w_octets, const float* x, size_t x_octets, const float* biais,
                 size_t biais_octets, float* y, size_t y_octets, uint32_t lignes, uint32_t colonnes, void* flux) {
    if (lignes == 0 || colonnes == 0 || colonnes % 4 != 0) return usage("shape %u x %u", lignes, colonnes);
    if (w == nullptr || w_octets < 4ull * lignes * colonnes || !aligne(w, 16)) return usage("f32 matrix too short or not aligned on 16");
    if (x == nullptr || x_octets < 4ull * colonnes || !aligne(x, 16)) return usage("x too short or not aligned on 16");
    if (y == nullptr || y_octets < 4ull * lignes) return usage("y too short");
    if (biais != nullptr && biais_octets < 4ull * lignes) return usage("bias too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_gemv_f32(w, x, 0, biais, y, lignes, colonnes, static_cast<cudaStream_t>(flux)));
}

int trc_routeur_topk(const float* logits, size_t logits_octets, uint32_t experts, uint32_t k, uint32_t* indices,
                     size_t indices_octets, float* poids, size_t poids_octets, uint64_t boite, uint32_t sequence,
                     void* flux) {
    if (experts == 0 || experts > 256 || k == 0 || k > 8 || k > experts) return usage("top-%u of %u", k, experts);
    if (logits == nullptr || logits_octets < 4ull * experts || indices == nullptr || indices_octets < 4ull * k ||
        poids == nullptr || poids_octets < 4ull * k)
        return usage("router: buffers too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_topk(logits, experts, k, indices, poids, reinterpret_cast<uint32_t*>(boite), sequence,
                                  static_cast<cudaStream_t>(flux)));
}

int trc_swiglu_oai(const float* g, size_t g_octets, const float* u, size_t u_octets, float* y, size_t y_octets,
                   uint32_t n, void* flux) {
    const uint64_t o = 4ull * n;
    if (n == 0 || g == nullptr || u == nullptr || y == nullptr || g_octets < o || u_octets < o || y_octets < o)
        return usage("swiglu: buffers too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_swiglu(g, u, y, n, static_cast<cudaStream_t>(flux)));
}

int trc_combiner(float* residu, size_t residu_octets, const float* sorties, size_t sorties_octets, uint32_t pas,
                 const float* poids, size_t poids_octets, uint32_t n, uint32_t d, void* flux) {
    if (n == 0 || d == 0 || (n > 1 && pas < d)) return usage("combine %u outputs of %u (stride %u)", n, d, pas);
    if (residu == nullptr || residu_octets < 4ull * d || sorties == nullptr ||
        sorties_octets < 4ull * ((uint64_t(n) - 1) * pas + d))
        return usage("combine: buffers too short");
    if (poids != nullptr && poids_octets < 4ull * n) return usage("weights too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_combiner(residu, sorties, pas, poids, n, d, static_cast<cudaStream_t>(flux)));
}

uint64_t trc_coder_flux_gpu_espace(uint32_t P, uint32_t N) {
    if (N == 0) return 0;
    return tb::coder_flux_espace(P, N);
}

int trc_coder_flux_gpu(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, uint32_t n_kappa,
                       const uint16_t* freqs, uint32_t n_tables, uint8_t* sortie, size_t capacite, uint64_t* octets,
                       void* espace, size_t espace_octets, void* flux) {
    if (P == 0 || P % 128 != 0 || N == 0 || N > 65535) return usage("P = %u (a multiple of 128), N = %u", P, N);
    if ((uint64_t(P) / 128 + N - 1) / N > 65535) return usage("more than 65,535 tiles");
    if (n_tables == 0 || n_tables > 4) return usage("%u tables (1 to 4)", n_tables);
    if (src == nullptr || !aligne(src, 4) || freqs == nullptr || !aligne(freqs, 2) || sortie == nullptr ||
        !aligne(sortie, 16) || octets == nullptr || !aligne(octets, 8))
        return usage("encoder: a buffer is missing or misaligned");
    if (kappa == nullptr && n_kappa != 0) return usage("contexts absent");
    if (espace == nullptr || !aligne(espace, 256) || espace_octets < tb::coder_flux_espace(P, N))
        return usage("encoder scratch of %zu bytes, %llu needed (256-aligned)", espace_octets,
                     (unsigned long long)tb::coder_flux_espace(P, N));
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_coder_flux(src, P, N, kappa, n_kappa, freqs, n_tables, sortie, capacite, octets,
                                        static_cast<uint8_t*>(espace), static_cast<cudaStream_t>(flux)));
}

static_assert(sizeof(trc_desc_codage) == 72 && sizeof(tb::DescCodage) == 72, "trc_desc_codage layout");

namespace {

int sms_du_device() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

int verifier_lot_codage(const trc_desc_codage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims) {
    if (const int r = verifier_dims(dims)) return r;
    if (n == 0 || n > 65535) return usage("%u experts (1 to 65,535)", n);
    if (descs == nullptr || !aligne(descs, 8) || descs_octets < sizeof(trc_desc_codage) * size_t(n))
        return usage("descriptors: %zu bytes for %u experts, or misaligned", descs_octets, n);
    return TRC_OK;
}

}  // namespace

uint64_t trc_coder_parties_gpu_espace(const trc_dims_expert* dims, uint32_t n, uint32_t n_delta, uint32_t n_codes) {
    if (dims == nullptr || n == 0 || n_delta == 0 || n_codes == 0) return 0;
    return tb::coder_parties_espace(dims_de(dims), n, n_delta, n_codes);
}

int trc_coder_parties_gpu(const trc_desc_codage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims,
                          const uint16_t* freqs, int canonique, uint16_t couche, uint32_t n_delta, uint32_t n_codes,
                          uint64_t* octets, size_t octets_octets, void* espace, size_t espace_octets, void* flux) {
    if (const int r = verifier_lot_codage(descs, descs_octets, n, dims)) return r;
    if (n_delta == 0 || n_delta > 65535 || n_codes == 0 || n_codes > 65535)
        return usage("tiles of %u / %u macro-steps (1 to 65,535)", n_delta, n_codes);
    for (int j = 0; j < 3; ++j) {
        const uint64_t nb = uint64_t(dims->lignes[j]) * (dims->colonnes[j] / 32);
        if ((nb + 127) / 128 / n_delta >= 65535 || (16 * nb + 127) / 128 / n_codes >= 65535)
            return usage("matrix %d: more than 65,535 tiles", j);
    }
    if (freqs == nullptr || !aligne(freqs, 2)) return usage("tables absent or misaligned");
    if (octets == nullptr || !aligne(octets, 8) || octets_octets < 16ull * n) return usage("octets: u64[2n] needed");
    const uint64_t besoin = tb::coder_parties_espace(dims_de(dims), n, n_delta, n_codes);
    if (espace == nullptr || !aligne(espace, 256) || espace_octets < besoin)
        return usage("encoder scratch of %zu bytes, %llu needed (256-aligned)", espace_octets, (unsigned long long)besoin);
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_coder_parties(reinterpret_cast<const tb::DescCodage*>(descs), n, dims_de(dims), freqs,
                                           canonique != 0, couche, n_delta, n_codes, octets,
                                           static_cast<uint8_t*>(espace), sms_du_device(), static_cast<cudaStream_t>(flux)));
}

int trc_comptes_gpu(const trc_desc_codage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims,
                    int canonique, uint64_t* comptes, size_t comptes_octets, void* flux) {
    if (const int r = verifier_lot_codage(descs, descs_octets, n, dims)) return r;
    if (comptes == nullptr || !aligne(comptes, 8) || comptes_octets < 3 * 4 * 256 * 8) return usage("counts: u64[3][4][256] needed");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_comptes(reinterpret_cast<const tb::DescCodage*>(descs), n, dims_de(dims), canonique != 0,
                                     comptes, sms_du_device(), static_cast<cudaStream_t>(flux)));
}

uint64_t trc_echange_octets(const trc_dims_expert* dims, uint32_t jetons, uint32_t monde) {
    if (dims == nullptr || monde == 0) return 0;
    return tb::disposition_echange(dims->lignes[2], jetons ? jetons : 1u, monde).total;
}

namespace {

// The descriptor's checks (Noyaux's usage rules for the layer's launches) and its translation.
// Tokens per call: 128 for the fused layer; a batch of positions par flux takes up to 4,096.
constexpr uint32_t JETONS_MAX = 128, JETONS_MAX_PAR_FLUX = 4096;

int couche_de(const trc_moe_couche* c, tb::Couche& k, uint32_t jetons_max = JETONS_MAX) {
    if (c == nullptr) return usage("layer descriptor absent");
    if (int s = verifier_dims(&c->dims)) return s;
    const trc_dims_expert& d = c->dims;
    if (c->k == 0 || c->k > 8 || c->k > c->experts) return usage("k = %u of %u experts", c->k, c->experts);
    const uint32_t jetons = c->jetons ? c->jetons : 1u;
    if (jetons > jetons_max) return usage("%u tokens (%u at most)", jetons, jetons_max);
    if (c->expert_fin != 0 && (c->expert_debut >= c->expert_fin || c->expert_fin > c->experts))
        return usage("held experts [%u, %u) of %u", c->expert_debut, c->expert_fin, c->experts);
    if (d.lignes[0] != d.lignes[1] || d.colonnes[0] != d.colonnes[1] || d.colonnes[2] != d.lignes[0] ||
        d.lignes[2] != d.colonnes[0])
        return usage("gate/up/down shapes do not chain (hidden -> ffn -> hidden)");
    for (int j = 0; j < 3; ++j) {
        if (d.colonnes[j] > 32768) return usage("matrix %d: %u columns (32,768 at most)", j, d.colonnes[j]);
        if (!c->brut && d.colonnes[j] < 256) return usage("matrix %d: %u columns (256 at least)", j, d.colonnes[j]);
        if (!c->brut && d.lignes[j] > 8192) return usage("matrix %d: %u rows (8,192 at most)", j, d.lignes[j]);
    }
    if (c->parties == nullptr || c->parties_octets == nullptr || c->indices == nullptr || c->poids == nullptr ||
        c->x == nullptr || c->residu == nullptr || c->controle == nullptr || (!c->brut && c->luts == nullptr))
        return usage("layer descriptor: a device buffer is missing");
    if (!aligne(c->x, c->x_bf16 ? 2 : 4)) return usage("x misaligned");
    if (!c->brut && !aligne(c->luts, 16)) return usage("LUTs misaligned (16 bytes)");
    k = tb::Couche{};
    k.parties = c->parties;
    k.parties_octets = c->parties_octets;
    k.experts = c->experts;
    k.k = c->k;
    k.luts = c->luts;
    for (int j = 0; j < 3; ++j) {
        k.lignes[j] = d.lignes[j];
        k.colonnes[j] = d.colonnes[j];
    }
    k.indices = c->indices;
    k.poids = c->poids;
    k.x = c->x;
    k.x_bf16 = c->x_bf16 ? 1u : 0u;
    k.brut = c->brut ? 1u : 0u;
    k.residu = c->residu;
    k.controle = c->controle;
    k.n_delta = c->n_delta;
    k.n_codes = c->n_codes;
    k.jetons = jetons;
    k.expert_debut = c->expert_debut;
    k.expert_fin = c->expert_fin;
    k.partiel = c->partiel ? 1u : 0u;
    k.deltas = c->brut ? nullptr : c->deltas;
    if (c->echange != nullptr) {
        const trc_echange_pairs& e = *c->echange;
        if (e.monde < 2 || e.monde > 8 || e.rang >= e.monde) return usage("exchange: rank %u of %u", e.rang, e.monde);
        if (c->partiel) return usage("exchange and partial combine together");
        for (uint32_t q = 0; q < e.monde; ++q) {
            if (e.tampons[q] == 0 || (e.tampons[q] & 255u) != 0) return usage("exchange buffer of rank %u absent or not 256-aligned", q);
            k.ech.tampons[q] = e.tampons[q];
        }
        k.ech.rang = e.rang;
        k.ech.monde = e.monde;
    }
    return TRC_OK;
}

}  // namespace

uint64_t trc_moe_espace_octets(const trc_dims_expert* dims, uint32_t k) {
    if (dims == nullptr || k == 0) return 0;
    return tb::plan_espace(dims->lignes, dims->colonnes, k).total;
}

uint64_t trc_moe_espace_recouvrant_octets(const trc_dims_expert* dims, uint32_t k) {
    if (dims == nullptr || k == 0) return 0;
    const tb::Espace e = tb::plan_espace(dims->lignes, dims->colonnes, k);
    return k <= tb::RECOUVRE_MAX ? e.total_tout : e.total;
}

uint64_t trc_gemm_mxfp4_espace_octets(uint32_t colonnes, uint32_t n) {
    if (colonnes == 0 || colonnes % 32 || n == 0 || n > 256) return 0;
    return tb::gemm_mxfp4_espace(colonnes, n);
}

int trc_gemm_mxfp4(const uint8_t* codes, const uint8_t* echelles, const float* biais, uint32_t lignes, uint32_t colonnes,
                   const void* x, uint32_t x_bf16, uint32_t n, float* y, void* espace, size_t espace_octets,
                   uint32_t* erreur, void* flux) {
    if (lignes == 0 || colonnes == 0 || colonnes % 32) return usage("%u x %u matrix (columns a multiple of 32)", lignes, colonnes);
    if (n == 0 || n > 256) return usage("%u tokens (1 to 256)", n);
    if (codes == nullptr || echelles == nullptr || x == nullptr || y == nullptr || espace == nullptr || erreur == nullptr)
        return usage("gemm: a device buffer is missing");
    if (!aligne(codes, 16) || !aligne(echelles, 16) || !aligne(espace, 256) || !aligne(x, x_bf16 ? 2 : 4) ||
        !aligne(y, 4))
        return usage("gemm: codes and scales 16-aligned, workspace 256-aligned");
    if (!tb::gemm_mxfp4_possible(colonnes, n)) return usage("gemm: %u columns x %u tokens exceed shared memory", colonnes, n);
    if (espace_octets < tb::gemm_mxfp4_espace(colonnes, n))
        return usage("gemm workspace of %zu bytes, %llu needed", espace_octets,
                     (unsigned long long)tb::gemm_mxfp4_espace(colonnes, n));
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_gemm_mxfp4(codes, echelles, biais, x, x_bf16 ? 1u : 0u, y, lignes, colonnes, n,
                                        static_cast<uint8_t*>(espace), erreur, static_cast<cudaStream_t>(flux)));
}

uint64_t trc_gemm_mxfp4_lot_espace_octets(uint32_t colonnes_max, uint32_t n_max, uint32_t nb) {
    if (colonnes_max == 0 || colonnes_max % 32 || n_max == 0 || n_max > 256 || nb == 0) return 0;
    return tb::gemm_mxfp4_lot_espace(colonnes_max, n_max, nb);
}

int trc_gemm_mxfp4_lot(const trc_desc_gemm* descs, uint32_t nb, uint32_t lignes_max, uint32_t colonnes_max,
                       uint32_t n_max, void* espace, size_t espace_octets, uint32_t* erreur, void* flux) {
    static_assert(sizeof(trc_desc_gemm) == sizeof(tb::DescGemm), "trc_desc_gemm layout");
    if (descs == nullptr || nb == 0 || nb > 65535) return usage("%u GEMM descriptors", nb);
    if (lignes_max == 0 || colonnes_max == 0 || colonnes_max % 32) return usage("%u x %u at most", lignes_max, colonnes_max);
    if (n_max == 0 || n_max > 256) return usage("%u tokens at most (1 to 256)", n_max);
    for (uint32_t i = 0; i < nb; ++i) {
        const trc_desc_gemm& d = descs[i];
        if (d.lignes == 0 || d.lignes > lignes_max || d.colonnes == 0 || d.colonnes % 32 || d.colonnes > colonnes_max ||
            d.n == 0 || d.n > n_max)
            return usage("gemm batch: matrix %u is %u x %u with %u tokens (at most %u x %u, %u tokens)", i, d.lignes,
                         d.colonnes, d.n, lignes_max, colonnes_max, n_max);
        if (d.codes == 0 || d.echelles == 0 || d.x == 0 || d.y == 0 || d.codes % 16 || d.echelles % 16 ||
            d.x % (d.x_bf16 ? 2 : 4) || d.y % 4)
            return usage("gemm batch: matrix %u: a buffer missing or misaligned (codes and scales 16-aligned)", i);
    }
    if (!tb::gemm_mxfp4_possible(colonnes_max, n_max))
        return usage("gemm batch: %u columns x %u tokens exceed shared memory", colonnes_max, n_max);
    if (espace == nullptr || erreur == nullptr || !aligne(espace, 256)) return usage("gemm batch: workspace 256-aligned");
    if (espace_octets < tb::gemm_mxfp4_lot_espace(colonnes_max, n_max, nb))
        return usage("gemm batch workspace of %zu bytes, %llu needed", espace_octets,
                     (unsigned long long)tb::gemm_mxfp4_lot_espace(colonnes_max, n_max, nb));
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_gemm_mxfp4_lot(reinterpret_cast<const tb::DescGemm*>(descs), nb, lignes_max, colonnes_max, n_max,
                                            static_cast<uint8_t*>(espace), erreur, static_cast<cudaStream_t>(flux)));
}

uint64_t trc_moe_deltas_octets(const trc_dims_expert* dims, uint32_t experts) {
    if (dims == nullptr || experts == 0) return 0;
    return tb::deltas_octets(dims->lignes, dims->colonnes, experts);
}

int trc_moe_predecoder_deltas(const trc_moe_couche* c, uint8_t* deltas, uint64_t deltas_octets, uint32_t* controle,
                              void* flux) {
    if (c == nullptr) return usage("layer descriptor absent");
    if (int s = verifier_dims(&c->dims)) return s;
    if (c->experts == 0) return usage("no expert");
    for (int j = 0; j < 3; ++j)
        if (c->dims.colonnes[j] < 256 || c->dims.lignes[j] > 8192)
            return usage("matrix %d: %u x %u (rows <= 8,192, columns >= 256)", j, c->dims.lignes[j], c->dims.colonnes[j]);
    if (c->parties == nullptr || c->parties_octets == nullptr || c->luts == nullptr || controle == nullptr ||
        deltas == nullptr)
        return usage("predecode: a device buffer is missing");
    if (!aligne(c->luts, 16)) return usage("LUTs misaligned (16 bytes)");
    const uint64_t besoin = tb::deltas_octets(c->dims.lignes, c->dims.colonnes, c->experts);
    if (deltas_octets < besoin) return usage("delta buffer of %llu bytes, %llu needed", (unsigned long long)deltas_octets,
                                             (unsigned long long)besoin);
    tb::Couche k{};
    k.parties = c->parties;
    k.parties_octets = c->parties_octets;
    k.experts = c->experts;
    k.k = 1;
    k.luts = c->luts;
    for (int j = 0; j < 3; ++j) {
        k.lignes[j] = c->dims.lignes[j];
        k.colonnes[j] = c->dims.colonnes[j];
    }
    k.controle = controle;
    k.n_delta = c->n_delta;
    k.jetons = 1;
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_predecoder_deltas(k, deltas, static_cast<cudaStream_t>(flux)));
}

int trc_moe_couche_fusionnee(const trc_moe_couche* c, void* espace, size_t espace_octets, void* flux) {
    return trc_moe_couche_chrono(c, espace, espace_octets, flux, nullptr);
}

int trc_moe_couche_chrono(const trc_moe_couche* c, void* espace, size_t espace_octets, void* flux,
                          void* const* evenements) {
    tb::Couche k;
    if (const int r = couche_de(c, k)) return r;
    const uint64_t besoin = tb::plan_espace(k.lignes, k.colonnes, c->k * k.jetons).total;
    if (espace == nullptr || espace_octets < besoin || !aligne(espace, 256))
        return usage("workspace of %zu bytes, %llu needed (256-aligned)", espace_octets, (unsigned long long)besoin);
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_moe(k, espace, espace_octets, static_cast<cudaStream_t>(flux),
                                 reinterpret_cast<cudaEvent_t const*>(evenements)));
}

uint64_t trc_moe_par_flux_espace_octets(const trc_dims_expert* dims, uint32_t experts, uint32_t activations) {
    if (dims == nullptr || experts == 0 || activations == 0) return 0;
    return tb::plan_par_flux(dims->lignes, dims->colonnes, experts, activations).total;
}

int trc_moe_couche_par_flux(const trc_moe_couche* c, void* espace, size_t espace_octets, void* flux) {
    tb::Couche k;
    if (const int r = couche_de(c, k, JETONS_MAX_PAR_FLUX)) return r;
    if (k.experts > 1024) return usage("par flux: %u experts (1,024 at most)", k.experts);
    if (k.ech.monde != 0) return usage("par flux: no exchange (an expert share with partiel is accepted)");
    const uint64_t besoin = tb::plan_par_flux(k.lignes, k.colonnes, k.experts, k.k * k.jetons).total;
    if (espace == nullptr || espace_octets < besoin || !aligne(espace, 256))
        return usage("workspace of %zu bytes, %llu needed (256-aligned)", espace_octets, (unsigned long long)besoin);
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_par_flux(k, espace, static_cast<cudaStream_t>(flux)));
}

uint64_t trc_moe_par_flux_mma_espace_octets(const trc_dims_expert* dims, uint32_t experts, uint32_t activations,
                                            uint32_t seuil) {
    if (dims == nullptr || experts == 0 || activations == 0 || seuil == 0) return 0;
    return tb::par_flux_mma_octets(dims->lignes, dims->colonnes, experts, activations, seuil);
}

int trc_moe_couche_par_flux_mma(const trc_moe_couche* c, uint32_t seuil, void* espace, size_t espace_octets,
                                uint32_t* erreur, void* flux) {
    tb::Couche k;
    if (const int r = couche_de(c, k, JETONS_MAX_PAR_FLUX)) return r;
    if (k.experts > 1024) return usage("par flux: %u experts (1,024 at most)", k.experts);
    if (k.ech.monde != 0) return usage("par flux: no exchange (an expert share with partiel is accepted)");
    if (seuil == 0) return usage("par flux on the tensor cores: threshold 0 (at least 1 activation per expert)");
    if (erreur == nullptr) return usage("par flux on the tensor cores: error word absent");
    for (int j = 0; j < 3; ++j)
        if (!tb::gemm_mxfp4_possible(k.colonnes[j], 256))
            return usage("par flux on the tensor cores: matrix %d's %u columns exceed shared memory", j, k.colonnes[j]);
    const uint64_t besoin = tb::par_flux_mma_octets(k.lignes, k.colonnes, k.experts, k.k * k.jetons, seuil);
    if (espace == nullptr || espace_octets < besoin || !aligne(espace, 256))
        return usage("workspace of %zu bytes, %llu needed (256-aligned)", espace_octets, (unsigned long long)besoin);
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_par_flux_mma(k, espace, seuil, erreur, static_cast<cudaStream_t>(flux)));
}

// ---------------------------------------------------------------- attention side (lib.rs:291-381)

int trc_gemv_q8_0(const void* w, size_t w_octets, const float* x, size_t x_octets, const float* biais,
                  size_t biais_octets, float* y, size_t y_octets, uint32_t lignes, uint32_t colonnes, void* flux) {
    if (lignes == 0 || colonnes == 0 || colonnes % 32 != 0) return usage("shape %u x %u", lignes, colonnes);
    if (colonnes > 16384) return usage("%u columns (16,384 at most)", colonnes);
    const uint64_t octets = uint64_t(lignes) * (colonnes / 32) * 34;
    if (w == nullptr || w_octets < octets || !aligne(w, 16))
        return usage("Q8_0 matrix of %zu bytes, %llu needed (16-aligned)", w_octets, (unsigned long long)octets);
    if (x == nullptr || x_octets < 4ull * colonnes || !aligne(x, 16)) return usage("x too short or not aligned on 16");
    if (y == nullptr || y_octets < 4ull * lignes) return usage("y too short");
    if (biais != nullptr && biais_octets < 4ull * lignes) return usage("bias too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_gemv_q8_0(w, x, biais, y, lignes, colonnes, static_cast<cudaStream_t>(flux)));
}

int trc_rmsnorm(const float* x, size_t x_octets, const float* w, size_t w_octets, float* y, size_t y_octets, uint32_t n,
                uint32_t lignes, float eps, void* flux) {
    if (n == 0 || lignes == 0) return usage("rmsnorm of %u x %u", lignes, n);
    const uint64_t o = 4ull * n * lignes;
    if (x == nullptr || y == nullptr || w == nullptr || x_octets < o || y_octets < o || w_octets < 4ull * n)
        return usage("rmsnorm: views too short");
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_rmsnorm(x, w, y, n, lignes, eps, static_cast<cudaStream_t>(flux)));
}

int trc_rope_yarn(float* q, size_t q_octets, float* k, size_t k_octets, uint32_t tetes_q, uint32_t tetes_k,
                  uint32_t position, const trc_params_rope* p, void* flux) {
    if (p == nullptr) return usage("rope parameters absent");
    if (p->dim_tete == 0 || p->dim_tete % 2 != 0 || p->dim_tete > 128) return usage("head dimension %u", p->dim_tete);
    if (p->variante > 1) return usage("YaRN variant %u", p->variante);
    const uint64_t d = p->dim_tete;
    if ((tetes_q && (q == nullptr || q_octets < 4 * d * tetes_q)) || (tetes_k && (k == nullptr || k_octets < 4 * d * tetes_k)))
        return usage("rope: views too short");
    if (tetes_q + tetes_k == 0) return TRC_OK;
    tb::ParamsRope r{p->base, p->facteur, p->ctx_origine, p->beta_rapide, p->beta_lent, p->dim_tete, p->variante};
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_rope_yarn(q, k, tetes_q, tetes_k, position, r, static_cast<cudaStream_t>(flux)));
}

int trc_ecrire_kv(const float* k, size_t k_octets, const float* v, size_t v_octets, uint16_t* cache_k,
                  size_t cache_k_octets, uint16_t* cache_v, size_t cache_v_octets, uint32_t dkv, uint32_t case_kv,
                  void* flux) {
    if (dkv == 0) return usage("dkv is 0");
    const uint64_t fin = 2ull * (uint64_t(case_kv) + 1) * dkv;
    if (k == nullptr || v == nullptr || k_octets < 4ull * dkv || v_octets < 4ull * dkv) return usage("k or v too short");
    if (cache_k == nullptr || cache_v == nullptr || cache_k_octets < fin || cache_v_octets < fin)
        return usage("case %u outside the cache", case_kv);
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_ecrire_kv(k, v, cache_k, cache_v, dkv, case_kv, static_cast<cudaStream_t>(flux)));
}

int trc_attention(const float* q, size_t q_octets, const uint16_t* cache_k, size_t cache_k_octets, const uint16_t* cache_v,
                  size_t cache_v_octets, const float* puits, size_t puits_octets, float* sortie, size_t sortie_octets,
                  const trc_params_attention* p, void* flux) {
    if (p == nullptr) return usage("attention parameters absent");
    if (p->dim_tete != 64 || p->tetes_kv == 0 || p->tetes % p->tetes_kv != 0)
        return usage("heads %u / %u of dimension %u", p->tetes, p->tetes_kv, p->dim_tete);
    if (p->fin < p->debut || p->fin - p->debut > 8192) return usage("positions [%u, %u)", p->debut, p->fin);
    if (p->anneau != 0 && p->fin - p->debut > p->anneau) return usage("more positions than cases in the ring");
    const uint64_t cases = p->anneau ? p->anneau : p->fin;
    const uint64_t dkv = uint64_t(p->tetes_kv) * 64;
    if (cache_k == nullptr || cache_v == nullptr || cache_k_octets < 2 * cases * dkv || cache_v_octets < 2 * cases * dkv)
        return usage("cache too short");
    if (!aligne(cache_k, 16) || !aligne(cache_v, 16)) return usage("key or value cache not aligned on 16");
    if (q == nullptr || sortie == nullptr || puits == nullptr || q_octets < 256ull * p->tetes ||
        sortie_octets < 256ull * p->tetes || puits_octets < 4ull * p->tetes)
        return usage("attention: views too short");
    if (p->tetes == 0 || p->fin == p->debut) return TRC_OK;
    tb::ParamsAttention a{p->tetes, p->tetes_kv, p->dim_tete, p->debut, p->fin, p->anneau, p->echelle, p->reserve};
    SUR_LE_FLUX(flux);
    return statut(tb::lancer_attention(q, cache_k, cache_v, puits, sortie, a, static_cast<cudaStream_t>(flux)));
}

int trc_routeur(const float* wr, const float* br, const void* x, uint32_t x_bf16, uint32_t experts, uint32_t colonnes,
                uint32_t k, uint32_t jetons, float* logits, uint32_t* indices, float* poids, void* flux) {
    if (experts == 0 || experts > 256 || k == 0 || k > 8 || k > experts) return usage("top-%u of %u", k, experts);
    if (jetons == 0 || jetons > JETONS_MAX_PAR_FLUX) return usage("%u tokens (1 to %u)", jetons, JETONS_MAX_PAR_FLUX);
    if (colonnes == 0 || colonnes % 4 != 0) return usage("%u columns (a multiple of 4)", colonnes);
    if (wr == nullptr || !aligne(wr, 16) || x == nullptr || !aligne(x, x_bf16 ? 8 : 16) || logits == nullptr ||
        indices == nullptr || poids == nullptr)
        return usage("router: a buffer is missing or misaligned");
    SUR_LE_FLUX(flux);
    cudaStream_t s = static_cast<cudaStream_t>(flux);
    cudaError_t e = tb::lancer_gemv_f32(wr, x, x_bf16 ? 1u : 0u, br, logits, experts, colonnes, s, jetons);
    if (e == cudaSuccess) e = tb::lancer_topk(logits, experts, k, indices, poids, nullptr, 0, s, jetons);
    return statut(e);
}

}  // extern "C"
