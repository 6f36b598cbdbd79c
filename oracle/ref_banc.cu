// TEST INFRASTRUCTURE — C entry points for the reference's second, independent .trc encoder.
//
// The reference's bench (moteur/crates/trc-noyaux/banc/banc_k.cu) writes the part format from
// the specification alone, without the Rust codec: its geometry-1 rANS coder (banc_k.cu:277-321),
// its LUT builder (banc_k.cu:256-261) and its part assembler (banc_k.cu:412-446). This file
// compiles that source unchanged from the reference checkout (oracle/Makefile, target `ref`) and
// exposes those three host functions, so the tests can check that the oracle's encoder writes
// the same stream and part bytes from the same frequency tables. The bench's own table
// normalisation (banc_k.cu:216-254, greedy, deliberately unlike the Rust codec's) is not used.
#include "banc_shim.h"

#define main banc_main
#include "banc_k.cu"
#undef main

namespace {
Table table_de(const uint16_t* f) {
    Table t;
    uint32_t c = 0;
    t.vide = true;
    for (int s = 0; s < 256; ++s) {
        t.f[s] = f[s];
        t.c[s] = c;
        c += f[s];
        if (f[s]) t.vide = false;
    }
    return t;
}
}  // namespace

// Geometry-1 stream of P bytes (a multiple of 128) in tiles of N macro-steps; table of word w:
// kappa[w / 4] when kappa is given and w / 4 < n_kappa, else 0 (as the bench's coder_expert
// chooses it, banc_k.cu:489). Returns the stream's size, 0 when `cap` is too small.
extern "C" size_t refb_coder_g1(const uint8_t* src, uint32_t P, uint32_t N, const uint16_t* freqs, uint32_t n_tables,
                                const uint8_t* kappa, uint32_t n_kappa, uint8_t* out, size_t cap) {
    std::vector<Table> t(n_tables);
    for (uint32_t k = 0; k < n_tables; ++k) t[k] = table_de(freqs + 256u * k);
    auto ctx = [kappa, n_kappa](uint32_t w) { return (kappa != nullptr && (w >> 2) < n_kappa) ? (uint32_t)kappa[w >> 2] : 0u; };
    const std::vector<uint8_t> o = coder_g1(src, P, N, t.data(), ctx);
    if (o.size() > cap) return 0;
    memcpy(out, o.data(), o.size());
    return o.size();
}

extern "C" void refb_lut_g1(const uint16_t* freqs, uint32_t* lut) {
    const Table t = table_de(freqs);
    lut_g1(t, lut);
}

// Part of n streams (descs: sorte, matrice, contexte per stream; stream bytes back to back in
// `donnees`); returns its size, 0 when `cap` is too small.
extern "C" size_t refb_assembler_partie(uint16_t couche, uint16_t expert, uint32_t n, const uint8_t* descs,
                                        const uint32_t* longueurs, const uint32_t* produits, const uint8_t* donnees,
                                        uint8_t* out, size_t cap) {
    std::vector<FluxPartie> flux(n);
    size_t o = 0;
    for (uint32_t i = 0; i < n; ++i) {
        flux[i].sorte = descs[3 * i];
        flux[i].matrice = descs[3 * i + 1];
        flux[i].contexte = descs[3 * i + 2];
        flux[i].octets.assign(donnees + o, donnees + o + longueurs[i]);
        flux[i].produits = produits[i];
        o += longueurs[i];
    }
    const std::vector<uint8_t> p = assembler_partie(couche, expert, flux);
    if (p.size() > cap) return 0;
    memcpy(out, p.data(), p.size());
    return p.size();
}
