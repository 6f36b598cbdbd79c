// troncons_b200 — the expert-parallel MoE layer through the C-ABI, for a host with no PyTorch:
// a Rust engine or a C program holding one process per GPU and an NCCL communicator over them.
//
// The reference is single-GPU: its combine is `combiner` over the k routed experts
// (trc-noyaux/noyaux/passe.cuh:611-622, driven by trc-modele/src/lib.rs:533-553). Here each rank
// holds a contiguous share of the layer's experts (the descriptor's expert_debut / expert_fin),
// runs the fused layer on it with the partial combine (rank 0 adds its share's weighted sum into
// the residual, every other rank writes its share's sum alone), then one NCCL SUM all-reduce of
// the [tokens][d] f32 residual on the same stream leaves the whole layer's result on every rank.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, or the copy a host already loaded), so
// the library links no NCCL of its own and shares the host's. The helpers below let a host with
// no NCCL binding create the communicator: trc_nccl_id on one rank, the 128 bytes sent to the
// others by any means, trc_nccl_init on every rank.
#include <dlfcn.h>
#include <nccl.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/troncons_b200.h"
#include "noyaux.h"

namespace {

struct Nccl {
    void* lib = nullptr;
    ncclResult_t (*id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*detruire)(ncclComm_t) = nullptr;
    ncclResult_t (*rang)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*compte)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*texte)(ncclResult_t) = nullptr;
};

const Nccl* nccl() {
    static std::once_flag fait;
    static Nccl n;
    std::call_once(fait, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the host's, when loaded
        if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) return;
        Nccl m;
        m.lib = h;
        m.id = reinterpret_cast<decltype(m.id)>(dlsym(h, "ncclGetUniqueId"));
        m.init = reinterpret_cast<decltype(m.init)>(dlsym(h, "ncclCommInitRank"));
        m.detruire = reinterpret_cast<decltype(m.detruire)>(dlsym(h, "ncclCommDestroy"));
        m.rang = reinterpret_cast<decltype(m.rang)>(dlsym(h, "ncclCommUserRank"));
        m.compte = reinterpret_cast<decltype(m.compte)>(dlsym(h, "ncclCommCount"));
        m.all_reduce = reinterpret_cast<decltype(m.all_reduce)>(dlsym(h, "ncclAllReduce"));
        m.texte = reinterpret_cast<decltype(m.texte)>(dlsym(h, "ncclGetErrorString"));
        if (m.id && m.init && m.detruire && m.rang && m.compte && m.all_reduce && m.texte) n = m;
    });
    return n.lib != nullptr ? &n : nullptr;
}

int erreur_nccl(const Nccl* n, ncclResult_t r) {
    char m[256];
    snprintf(m, sizeof m, "NCCL: %s", n->texte(r));
    tb::erreur_usage(m);  // records the text
    return TRC_ERR_CUDA;
}

}  // namespace

extern "C" {

int trc_nccl_id(uint8_t* id, size_t id_octets) {
    const Nccl* n = nccl();
    if (n == nullptr) return tb::erreur_usage("libnccl.so.2 not found");
    if (id == nullptr || id_octets < NCCL_UNIQUE_ID_BYTES) return tb::erreur_usage("unique id: 128 bytes expected");
    ncclUniqueId u;
    if (ncclResult_t r = n->id(&u)) return erreur_nccl(n, r);
    memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
    return TRC_OK;
}

int trc_nccl_init(void** comm, uint32_t monde, const uint8_t* id, uint32_t rang) {
    const Nccl* n = nccl();
    if (n == nullptr) return tb::erreur_usage("libnccl.so.2 not found");
    if (comm == nullptr || id == nullptr || monde == 0 || rang >= monde) {
        char m[96];
        snprintf(m, sizeof m, "rank %u of %u, or a pointer absent", rang, monde);
        return tb::erreur_usage(m);
    }
    ncclUniqueId u;
    memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t c = nullptr;
    if (ncclResult_t r = n->init(&c, int(monde), u, int(rang))) return erreur_nccl(n, r);
    *comm = c;
    return TRC_OK;
}

int trc_nccl_fin(void* comm) {
    const Nccl* n = nccl();
    if (n == nullptr) return tb::erreur_usage("libnccl.so.2 not found");
    if (comm == nullptr) return TRC_OK;
    if (ncclResult_t r = n->detruire(static_cast<ncclComm_t>(comm))) return erreur_nccl(n, r);
    return TRC_OK;
}

int trc_moe_couche_ep(const trc_moe_couche* couche, void* espace, size_t espace_octets, void* comm, void* flux) {
    const Nccl* n = nccl();
    if (n == nullptr) return tb::erreur_usage("libnccl.so.2 not found");
    if (couche == nullptr || comm == nullptr) return tb::erreur_usage("layer descriptor or communicator absent");
    if (couche->partiel || couche->echange != nullptr)
        return tb::erreur_usage("expert-parallel layer: partiel and echange are set by the call itself");
    int rang = 0, monde = 0;
    if (ncclResult_t r = n->rang(static_cast<ncclComm_t>(comm), &rang)) return erreur_nccl(n, r);
    if (ncclResult_t r = n->compte(static_cast<ncclComm_t>(comm), &monde)) return erreur_nccl(n, r);
    trc_moe_couche c = *couche;
    c.partiel = rang != 0 ? 1u : 0u;
    if (int s = trc_moe_couche_fusionnee(&c, espace, espace_octets, flux)) return s;
    if (monde == 1) return TRC_OK;
    const size_t n_val = size_t(c.jetons ? c.jetons : 1u) * c.dims.lignes[2];
    if (ncclResult_t r = n->all_reduce(c.residu, c.residu, n_val, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm),
                                       static_cast<cudaStream_t>(flux)))
        return erreur_nccl(n, r);
    return TRC_OK;
}

}  // extern "C"
