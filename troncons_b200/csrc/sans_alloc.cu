// troncons_b200 — the fused MoE layer with no workspace argument, for callers that cannot
// allocate device memory when they run the layer. Such callers include a host binding with no
// device allocator of its own (a plain C or FFI caller that only holds pointers to buffers it was
// given), a serving loop whose device memory was fixed up front and must not grow, and code on a
// path where an allocation would synchronise the device or fail under memory pressure.
//
// The workspace is one area of this library's own device memory, declared below as a static
// device array of ESPACE_FIXE_OCTETS bytes, so it exists as soon as the library's module is
// loaded on a device; nothing here calls an allocator. Its address on a device is looked up once
// per device (the first call on that device, with the device current) and kept for the life of
// the process: after a cudaDeviceReset of that device the kept address is stale, so the entry
// point must not be called on a device that was reset since its first call there.
//
// Every call on a device uses the same area. Calls on one stream run one after another and are
// safe; calls that can overlap in time on one device (two streams, or two host threads with
// different streams) race on it and give wrong results: order them, or use
// trc_moe_couche_fusionnee with a workspace of each caller's own. Nothing in the area needs to
// start at zero: every byte a call reads from it was written earlier in that same call.
#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/troncons_b200.h"
#include "noyaux.h"

namespace {

// 8 MiB: the gpt-oss-120b expert shapes (2880 x 2880 gate/up/down) need 6,865,920 bytes at k = 8
// and 3,432,960 at k = 4.
constexpr size_t ESPACE_FIXE_OCTETS = size_t(8) << 20;

constexpr int DEVICES_MAX = 64;

}  // namespace

static __device__ __align__(256) uint8_t espace_fixe[ESPACE_FIXE_OCTETS];

namespace {

std::mutex verrou_adresses;
void* adresses[DEVICES_MAX] = {};

// The area's address on the current device, looked up on the first call for that device.
cudaError_t adresse_espace_fixe(void** p) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= DEVICES_MAX) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(verrou_adresses);
    if (adresses[dev] == nullptr) {
        void* a = nullptr;
        e = cudaGetSymbolAddress(&a, espace_fixe);
        if (e != cudaSuccess) return e;
        adresses[dev] = a;
    }
    *p = adresses[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int trc_moe_couche_sans_alloc(const trc_moe_couche* couche, void* flux) {
    if (couche == nullptr) return tb::erreur_usage("layer descriptor absent");
    // k and the token count first, with trc_moe_couche_fusionnee's rules and messages, so that a
    // bad one is reported as itself and not as a workspace size.
    char m[256];
    if (couche->k == 0 || couche->k > 8 || couche->k > couche->experts) {
        snprintf(m, sizeof m, "k = %u of %u experts", couche->k, couche->experts);
        return tb::erreur_usage(m);
    }
    const uint32_t jetons = couche->jetons ? couche->jetons : 1u;
    if (jetons > 128) {
        snprintf(m, sizeof m, "%u tokens (128 at most)", jetons);
        return tb::erreur_usage(m);
    }
    const uint64_t besoin = trc_moe_espace_octets(&couche->dims, couche->k * jetons);
    if (besoin > ESPACE_FIXE_OCTETS) {
        snprintf(m, sizeof m,
                 "layer needs %llu bytes of workspace; the fixed area holds %zu (use trc_moe_couche_fusionnee with a "
                 "workspace of its size)",
                 static_cast<unsigned long long>(besoin), ESPACE_FIXE_OCTETS);
        return tb::erreur_usage(m);
    }
    cudaError_t e = tb::aligner_device(flux);
    if (e != cudaSuccess) return tb::erreur_cuda(e);
    void* espace = nullptr;
    if ((e = adresse_espace_fixe(&espace)) != cudaSuccess) return tb::erreur_cuda(e);
    return trc_moe_couche_fusionnee(couche, espace, ESPACE_FIXE_OCTETS, flux);
}
