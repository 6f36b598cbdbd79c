// troncons_b200 — the streaming layer executor: MoE layers whose experts' parts live in host
// memory (a pinned tier, all of the model) and are brought to the GPU on demand into a pool of
// part slots that the expert cache manages (trc-ordo's on-demand step, moteur/crates/trc-ordo/
// src/lib.rs:1054-1367, with trc-cache, lib.rs:105-301).
//
// The reference copies a missing expert's part to an arrival buffer and decodes it into a slot
// of decoded weights; here the slot holds the part itself (the fused layer decodes while it
// multiplies), so a miss is one host-to-device copy. Per layer call:
//   1. the routed experts: imposed by the caller (a routing trace), or from the router on the
//      compute stream, read back and waited for on the host (the reference's mailbox + event);
//   2. the cache serves the layer's distinct experts (pins them, evicts unpinned present slots);
//   3. each miss: its part copied from the host tier into its slot on the copy stream, after the
//      last launch that read the slot's previous part (an event per layer call);
//   4. the layer's part table (addresses and sizes of its experts, 0 for absent ones) staged and
//      copied on the compute stream, which waits for the copies; then the fused layer;
//   5. misses marked ready, the layer released (the reference's order, lib.rs:1322-1330).
// The host runs at most RING layer calls ahead of the GPU (it waits for the event of the call
// RING back before reusing its staging buffers).
#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <vector>

#include "../../include/troncons_b200.h"
#include "commun.cuh"
#include "noyaux.h"

namespace {

constexpr uint32_t RING = 8;

// Up to three host-to-device moves in one launch, from mapped pinned memory: the layer's part
// table and the imposed routing. A kernel, not a copy: a copy on the compute stream would wait
// in the copy engine's queue behind the large part copies already issued for later layers.
struct Transferts {
    uint4* dst[3];
    const uint4* src[3];
    uint32_t n[3];  // 16-byte words
};

__global__ void __launch_bounds__(256) k_transferer(Transferts t) {
    for (int i = 0; i < 3; ++i)
        for (uint32_t w = threadIdx.x; w < t.n[i]; w += blockDim.x) t.dst[i][w] = t.src[i][w];
}

struct Disposition {
    uint64_t table, idx, poids, logits, controle, moe, total;
};

Disposition disposition(const trc_flux_config& c) {
    Disposition d{};
    const uint64_t na = uint64_t(c.jetons_max) * c.k;
    uint64_t p = 0;
    d.table = p;
    p = tb::al256(p + 16ull * c.couches * c.experts);
    d.idx = p;
    p = tb::al256(p + 4 * na);
    d.poids = p;
    p = tb::al256(p + 4 * na);
    d.logits = p;
    p = tb::al256(p + 4ull * c.jetons_max * c.experts);
    d.controle = p;
    p = tb::al256(p + 16 * na);
    d.moe = p;
    p = tb::al256(p + trc_moe_espace_recouvrant_octets(&c.dims, uint32_t(na)));
    d.total = p;
    return d;
}

}  // namespace

struct trc_flux {
    trc_flux_config c{};
    Disposition d{};
    trc_cache* cache = nullptr;
    cudaStream_t calcul = nullptr, copie = nullptr;
    cudaEvent_t fin[RING] = {}, copies[RING] = {}, routeur = nullptr;
    bool fin_utilise[RING] = {};
    uint8_t* hote = nullptr;  // mapped pinned staging: per ring entry [table 16 E][idx][poids] (16-aligned);
                              // then the router's indices read back
    uint8_t* hote_carte = nullptr;  // its device address
    uint64_t pas_hote = 0;
    uint64_t appel = 0, pas = 0;
    std::vector<int64_t> lecteur;  // per slot: the last call whose layer read it (-1: none)
    std::vector<uint64_t> adr_hote, tailles;

    ~trc_flux() {
        for (uint32_t i = 0; i < RING; ++i) {
            if (fin[i]) cudaEventDestroy(fin[i]);
            if (copies[i]) cudaEventDestroy(copies[i]);
        }
        if (routeur) cudaEventDestroy(routeur);
        if (copie) cudaStreamDestroy(copie);
        if (hote) cudaFreeHost(hote);
        if (cache) trc_cache_detruire(cache);
    }
};

namespace {

int usage(const char* m) { return tb::erreur_usage(m); }

}  // namespace

extern "C" {

uint64_t trc_flux_espace_octets(const trc_flux_config* c) {
    if (c == nullptr || c->k == 0 || c->jetons_max == 0) return 0;
    return disposition(*c).total;
}

trc_flux* trc_flux_nouveau(const trc_flux_config* c) {
    if (c == nullptr || c->couches == 0 || c->experts == 0 || c->experts > 65535 || c->couches > 65535 || c->k == 0 ||
        c->k > 8 || c->jetons_max == 0 || c->jetons_max > 128 || c->emplacements < c->k * c->jetons_max) {
        usage("streaming executor: layers, experts, k (1..8), tokens (1..128) or slots (>= k x tokens)");
        return nullptr;
    }
    if (c->taille_emplacement == 0 || c->taille_emplacement % 256 != 0 || c->emplacements_carte == 0 ||
        c->emplacements_carte % 256 != 0 || c->parties_hote == 0 || c->tailles_parties == 0 || c->luts == 0 ||
        c->espace == 0 || c->espace % 256 != 0) {
        usage("streaming executor: a buffer is missing or misaligned (slots and workspace 256-aligned)");
        return nullptr;
    }
    const uint64_t* tailles = reinterpret_cast<const uint64_t*>(c->tailles_parties);
    for (uint64_t i = 0; i < uint64_t(c->couches) * c->experts; ++i)
        if (tailles[i] > c->taille_emplacement) {
            usage("streaming executor: a part is larger than a slot");
            return nullptr;
        }
    if (cudaError_t e0 = tb::aligner_device(reinterpret_cast<void*>(c->flux))) {
        tb::erreur_cuda(e0);
        return nullptr;
    }
    auto* f = new trc_flux();
    f->c = *c;
    f->d = disposition(*c);
    f->calcul = reinterpret_cast<cudaStream_t>(c->flux);
    f->cache = trc_cache_nouveau(c->emplacements, 0, TRC_POLITIQUE_LRU, nullptr, 0, 0, 0, 0);
    f->lecteur.assign(c->emplacements, -1);
    f->adr_hote.assign(reinterpret_cast<const uint64_t*>(c->parties_hote),
                       reinterpret_cast<const uint64_t*>(c->parties_hote) + uint64_t(c->couches) * c->experts);
    f->tailles.assign(tailles, tailles + uint64_t(c->couches) * c->experts);
    const uint64_t na = uint64_t(c->jetons_max) * c->k;
    f->pas_hote = tb::al256(16ull * c->experts + 2 * ((4 * na + 15) / 16 * 16));
    cudaError_t e = cudaStreamCreateWithFlags(&f->copie, cudaStreamNonBlocking);
    for (uint32_t i = 0; i < RING && e == cudaSuccess; ++i) {
        e = cudaEventCreateWithFlags(&f->fin[i], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&f->copies[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&f->routeur, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaHostAlloc(&f->hote, f->pas_hote * RING + 4 * na, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&f->hote_carte), f->hote, 0);
    // The table starts empty (every address 0) and the integrity counters at 0.
    uint8_t* esp = reinterpret_cast<uint8_t*>(c->espace);
    if (e == cudaSuccess) e = cudaMemsetAsync(esp + f->d.table, 0, 16ull * c->couches * c->experts, f->calcul);
    if (e == cudaSuccess) e = cudaMemsetAsync(esp + f->d.controle, 0, 16 * na, f->calcul);
    if (e != cudaSuccess || f->cache == nullptr) {
        tb::erreur_cuda(e == cudaSuccess ? cudaErrorInvalidValue : e);
        delete f;
        return nullptr;
    }
    return f;
}

void trc_flux_detruire(trc_flux* f) { delete f; }

int trc_flux_couche(trc_flux* f, uint32_t couche, const void* x, uint32_t x_bf16, float* residu, uint32_t jetons,
                    const uint32_t* experts_imposes, const float* poids_imposes, trc_flux_stats* stats) {
    if (f == nullptr || couche >= f->c.couches || x == nullptr || residu == nullptr || jetons == 0 ||
        jetons > f->c.jetons_max || (experts_imposes == nullptr) != (poids_imposes == nullptr))
        return usage("streaming layer: layer, x, residual, tokens, or imposed experts without weights");
    if (experts_imposes == nullptr && (f->c.routeurs == 0 || f->c.biais_routeurs == 0))
        return usage("streaming layer: no router weights, and no imposed experts");
    if (cudaError_t e0 = tb::aligner_device(reinterpret_cast<void*>(f->c.flux))) return tb::erreur_cuda(e0);
    const trc_flux_config& c = f->c;
    const uint32_t na = jetons * c.k, E = c.experts;
    uint8_t* esp = reinterpret_cast<uint8_t*>(c.espace);
    uint32_t* idx_dev = reinterpret_cast<uint32_t*>(esp + f->d.idx);
    float* poids_dev = reinterpret_cast<float*>(esp + f->d.poids);
    const uint32_t r = uint32_t(f->appel % RING);
    uint8_t* st = f->hote + r * f->pas_hote;
    const uint64_t n16 = (4ull * na + 15) / 16;  // 16-byte words of idx, and of poids
    uint32_t* idx_st = reinterpret_cast<uint32_t*>(st + 16ull * E);
    float* poids_st = reinterpret_cast<float*>(st + 16ull * E + 16 * n16);
    uint8_t* st_carte = f->hote_carte + r * f->pas_hote;
    uint32_t* idx_lu = reinterpret_cast<uint32_t*>(f->hote + f->pas_hote * RING);
    trc_flux_stats s{};
    cudaError_t e;
    // Ring entry r was last used RING calls ago: its launches must be done before its staging
    // is rewritten.
    if (f->fin_utilise[r] && (e = cudaEventSynchronize(f->fin[r])) != cudaSuccess) return tb::erreur_cuda(e);

    // 1. the routed experts
    const uint32_t* experts;
    if (experts_imposes != nullptr) {
        for (uint32_t i = 0; i < na; ++i)
            if (experts_imposes[i] >= E) return usage("streaming layer: an imposed expert is out of range");
        std::memcpy(idx_st, experts_imposes, 4ull * na);
        std::memcpy(poids_st, poids_imposes, 4ull * na);
        experts = experts_imposes;  // moved to the device with the part table (step 4)
    } else {
        const float* wr = reinterpret_cast<const float*>(c.routeurs) + uint64_t(couche) * E * c.dims.colonnes[0];
        const float* br = reinterpret_cast<const float*>(c.biais_routeurs) + uint64_t(couche) * E;
        const int st2 = trc_routeur(wr, br, x, x_bf16, E, c.dims.colonnes[0], c.k, jetons,
                                    reinterpret_cast<float*>(esp + f->d.logits), idx_dev, poids_dev, f->calcul);
        if (st2 != TRC_OK) return st2;
        if ((e = cudaMemcpyAsync(idx_lu, idx_dev, 4ull * na, cudaMemcpyDeviceToHost, f->calcul)) != cudaSuccess ||
            (e = cudaEventRecord(f->routeur, f->calcul)) != cudaSuccess)
            return tb::erreur_cuda(e);
        const auto t0 = std::chrono::steady_clock::now();
        if ((e = cudaEventSynchronize(f->routeur)) != cudaSuccess) return tb::erreur_cuda(e);
        s.attente_routeur_s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        for (uint32_t i = 0; i < na; ++i)
            if (idx_lu[i] >= E) return usage("streaming layer: the router wrote an expert out of range");
        experts = idx_lu;
    }

    // 2. the layer's distinct experts, in first-appearance order, through the cache
    uint16_t uniques[8 * 128];
    uint32_t nu = 0;
    for (uint32_t i = 0; i < na; ++i) {
        bool vu = false;
        for (uint32_t j = 0; j < nu && !vu; ++j) vu = uniques[j] == experts[i];
        if (!vu) uniques[nu++] = uint16_t(experts[i]);
    }
    trc_decision dec[8 * 128];
    const uint64_t t = f->pas * c.couches + couche;
    if (int st3 = trc_cache_demander(f->cache, uint16_t(couche), uniques, nu, t, dec)) return st3;

    // 3. the misses' parts into their slots, each after the last launch that read the slot
    uint8_t* emplacements = reinterpret_cast<uint8_t*>(c.emplacements_carte);
    for (uint32_t j = 0; j < nu; ++j) {
        if (dec[j].sorte == TRC_DECISION_SUCCES) {
            ++s.succes;
            continue;
        }
        const uint64_t ie = uint64_t(couche) * E + uniques[j];
        const uint32_t sl = dec[j].emplacement;
        const int64_t l = f->lecteur[sl];
        if (l >= 0 && uint64_t(l) + RING > f->appel &&
            (e = cudaStreamWaitEvent(f->copie, f->fin[uint64_t(l) % RING], 0)) != cudaSuccess)
            return tb::erreur_cuda(e);
        if ((e = cudaMemcpyAsync(emplacements + uint64_t(sl) * c.taille_emplacement,
                                 reinterpret_cast<const void*>(f->adr_hote[ie]), f->tailles[ie], cudaMemcpyHostToDevice,
                                 f->copie)) != cudaSuccess)
            return tb::erreur_cuda(e);
        ++s.defauts;
        s.octets_copies += f->tailles[ie];
    }
    if ((e = cudaEventRecord(f->copies[r], f->copie)) != cudaSuccess ||
        (e = cudaStreamWaitEvent(f->calcul, f->copies[r], 0)) != cudaSuccess)
        return tb::erreur_cuda(e);

    // 4. the layer's part table, then the fused layer
    uint64_t* tab = reinterpret_cast<uint64_t*>(st);
    std::memset(tab, 0, 16ull * E);
    for (uint32_t j = 0; j < nu; ++j) {
        tab[uniques[j]] = uint64_t(c.emplacements_carte) + uint64_t(dec[j].emplacement) * c.taille_emplacement;
        tab[E + uniques[j]] = f->tailles[uint64_t(couche) * E + uniques[j]];
    }
    uint64_t* table_dev = reinterpret_cast<uint64_t*>(esp + f->d.table) + 2ull * couche * E;
    Transferts tr{};
    tr.dst[0] = reinterpret_cast<uint4*>(table_dev);
    tr.src[0] = reinterpret_cast<const uint4*>(st_carte);
    tr.n[0] = E;
    if (experts_imposes != nullptr) {
        tr.dst[1] = reinterpret_cast<uint4*>(idx_dev);
        tr.src[1] = reinterpret_cast<const uint4*>(st_carte + 16ull * E);
        tr.n[1] = uint32_t(n16);
        tr.dst[2] = reinterpret_cast<uint4*>(poids_dev);
        tr.src[2] = reinterpret_cast<const uint4*>(st_carte + 16ull * E + 16 * n16);
        tr.n[2] = uint32_t(n16);
    }
    k_transferer<<<1, 256, 0, f->calcul>>>(tr);
    if ((e = cudaGetLastError()) != cudaSuccess) return tb::erreur_cuda(e);
    trc_moe_couche m{};
    m.parties = table_dev;
    m.parties_octets = table_dev + E;
    m.experts = E;
    m.k = c.k;
    m.luts = reinterpret_cast<const uint32_t*>(c.luts) + uint64_t(couche) * 3 * 4 * 4096;
    m.dims = c.dims;
    m.indices = idx_dev;
    m.poids = poids_dev;
    m.x = x;
    m.x_bf16 = x_bf16;
    m.residu = residu;
    m.controle = reinterpret_cast<uint32_t*>(esp + f->d.controle);
    m.n_delta = c.n_delta;
    m.n_codes = c.n_codes;
    m.jetons = jetons;
    if (int st4 = trc_moe_couche_fusionnee(&m, esp + f->d.moe, f->d.total - f->d.moe, f->calcul)) return st4;
    if ((e = cudaEventRecord(f->fin[r], f->calcul)) != cudaSuccess) return tb::erreur_cuda(e);
    f->fin_utilise[r] = true;
    for (uint32_t j = 0; j < nu; ++j) f->lecteur[dec[j].emplacement] = int64_t(f->appel);

    // 5. ready, released
    for (uint32_t j = 0; j < nu; ++j)
        if (dec[j].sorte != TRC_DECISION_SUCCES)
            if (int st5 = trc_cache_pret(f->cache, dec[j].emplacement)) return st5;
    trc_cache_liberer(f->cache, uint16_t(couche));
    s.uniques = nu;
    if (stats != nullptr) *stats = s;
    ++f->appel;
    if (couche + 1 == c.couches) ++f->pas;
    return TRC_OK;
}

int trc_flux_compteurs(const trc_flux* f, trc_compteurs_cache* sortie) {
    if (f == nullptr || sortie == nullptr) return usage("streaming executor absent");
    trc_cache_compteurs(f->cache, sortie);
    return TRC_OK;
}

int trc_flux_controle(const trc_flux* f, uint32_t* sortie, uint32_t n) {
    if (f == nullptr || sortie == nullptr) return usage("streaming executor absent");
    const uint32_t na = f->c.jetons_max * f->c.k;
    const uint32_t m = n < 4 * na ? n : 4 * na;
    const cudaError_t e = cudaMemcpy(sortie, reinterpret_cast<const uint8_t*>(f->c.espace) + f->d.controle, 4ull * m,
                                     cudaMemcpyDeviceToHost);
    return e == cudaSuccess ? TRC_OK : tb::erreur_cuda(e);
}

}  // extern "C"
