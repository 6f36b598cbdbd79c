// troncons_b200 — the host side of the `.trc` format: LUTs of a layer, the v1.0/v1.2 encoder of
// an expert part (what `trc-codeur coder [--canonique|--brut]` writes), and a seeded generator of
// synthetic MXFP4 experts. Multi-threaded where it pays (per matrix / per row).
//
// Reference: trc-codec/src/rans.rs (tables 83-166, coder 296-334), trc-codec/src/lib.rs
// (preparer_matrice_avec 348-373, ComptesMatrice 377-413, coder_matrice_v10 417-428, flux_bruts
// 432-445), trc-format/src/lib.rs (canonical bytes 67-83, assembler_partie 882-908),
// bins/trc-codeur/src/coder.rs:243-313 (stream order per part).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

#include "../../include/troncons_b200.h"

namespace {

constexpr uint32_t M = 4096, L = 65536;

void eu16(uint8_t* p, uint32_t v) {
    p[0] = uint8_t(v);
    p[1] = uint8_t(v >> 8);
}
void eu32(uint8_t* p, uint32_t v) {
    for (int i = 0; i < 4; ++i) p[i] = uint8_t(v >> (8 * i));
}

uint8_t canonique_octet(uint8_t o) {
    uint8_t lo = o & 15, hi = o >> 4;
    if (lo == 8) lo = 0;
    if (hi == 8) hi = 0;
    return uint8_t(lo | (hi << 4));
}

uint8_t classe(uint8_t d) { return d < 128 ? 0 : (d == 128 ? 1 : 2); }

// Medians, padded delta and padded qs of one matrix (lib.rs:348-373).
struct Prepa {
    std::vector<uint8_t> med, delta, qs;
};

Prepa preparer(const uint8_t* blocs, uint32_t R, uint32_t B, bool canonique) {
    const size_t nb = size_t(R) * B;
    Prepa p;
    p.med.resize(R);
    p.delta.assign((nb + 127) / 128 * 128, 0);
    p.qs.assign((16 * nb + 127) / 128 * 128, 0);
    std::vector<uint8_t> tri(B);
    for (uint32_t r = 0; r < R; ++r) {
        const uint8_t* ligne = blocs + size_t(r) * B * 17;
        for (uint32_t b = 0; b < B; ++b) tri[b] = ligne[17 * b];
        std::nth_element(tri.begin(), tri.begin() + B / 2, tri.end());
        const uint8_t med = tri[B / 2];
        p.med[r] = med;
        for (uint32_t b = 0; b < B; ++b) {
            const size_t beta = size_t(r) * B + b;
            p.delta[beta] = uint8_t(ligne[17 * b] - med + 128);
            std::memcpy(&p.qs[16 * beta], ligne + 17 * b + 1, 16);
        }
    }
    if (canonique)
        for (auto& q : p.qs) q = canonique_octet(q);
    return p;
}

// Geometry-1 encoder of `src` (a multiple of 128 bytes) with N macro-steps per tile; table of
// byte n: kappa[n / 16] when kappa is given (0 beyond it), else table 0 (rans.rs:296-334).
std::vector<uint8_t> coder_g1(const std::vector<uint8_t>& src, uint32_t N, const std::vector<uint8_t>* kappa,
                              const uint16_t* const* freqs) {
    const uint32_t P = uint32_t(src.size());
    const uint32_t nmacro = P / 128, T = (nmacro + N - 1) / N;
    uint32_t cumul[3][256];
    const int ntab = kappa ? 3 : 1;
    for (int t = 0; t < ntab; ++t) {
        uint32_t c = 0;
        for (int s = 0; s < 256; ++s) {
            cumul[t][s] = c;
            c += freqs[t][s];
        }
    }
    std::vector<uint32_t> debut(T), etats(32ull * T);
    std::vector<uint16_t> mots, pile;
    mots.reserve(P / 2 + 64);
    for (uint32_t t = 0; t < T; ++t) {
        const uint32_t m0 = t * N, m1 = std::min(m0 + N, nmacro);
        uint64_t x[32];
        for (auto& v : x) v = L;
        pile.clear();
        for (uint32_t m = m1; m-- > m0;) {
            for (int k = 3; k >= 0; --k) {
                for (int l = 31; l >= 0; --l) {
                    const size_t n = (size_t(m) * 32 + l) * 4 + k;
                    const int c = kappa ? (n / 16 < kappa->size() ? (*kappa)[n / 16] : 0) : 0;
                    const uint32_t s = src[n];
                    const uint64_t f = freqs[c][s];
                    if (f == 0) return {};  // a symbol absent from its table: the caller's error
                    uint64_t xv = x[l];
                    if (xv >= (f << 20)) {
                        pile.push_back(uint16_t(xv & 0xFFFF));
                        xv >>= 16;
                    }
                    x[l] = ((xv / f) << 12) + (xv % f) + cumul[c][s];
                }
            }
        }
        debut[t] = uint32_t(mots.size());
        for (int l = 0; l < 32; ++l) etats[32ull * t + l] = uint32_t(x[l]);
        mots.insert(mots.end(), pile.rbegin(), pile.rend());
    }
    const uint32_t W = uint32_t(mots.size());
    std::vector<uint8_t> o((16 + 4ull * T + 128ull * T + 2ull * W + 15) / 16 * 16, 0);
    eu32(&o[0], P);
    eu16(&o[4], N);
    o[6] = 1;
    o[7] = 0;
    eu32(&o[8], T);
    eu32(&o[12], W);
    std::memcpy(&o[16], debut.data(), 4ull * T);
    std::memcpy(&o[16 + 4ull * T], etats.data(), 128ull * T);
    std::memcpy(&o[16 + 132ull * T], mots.data(), 2ull * W);
    return o;
}

struct FluxP {
    uint8_t sorte, matrice, contexte;
    uint32_t produits;
    std::vector<uint8_t> octets;
};

// Part assembly (trc-format/src/lib.rs:882-908). Returns the part length; writes it if it fits.
int64_t assembler(uint16_t couche, uint16_t expert, const std::vector<FluxP>& flux, uint8_t* sortie, size_t capacite,
                  uint32_t* utiles_out) {
    const size_t n = flux.size();
    size_t p = 64 + 16 * n;
    std::vector<size_t> dec(n);
    for (size_t i = 0; i < n; ++i) {
        p = (p + 15) / 16 * 16;
        dec[i] = p;
        p += flux[i].octets.size();
    }
    const size_t utiles = p, total = (utiles + 4095) / 4096 * 4096;
    if (utiles_out) *utiles_out = uint32_t(utiles);
    if (sortie == nullptr || capacite < total) return int64_t(total);
    std::memset(sortie, 0, total);
    eu32(sortie, 0x30435254u);
    eu16(sortie + 4, couche);
    eu16(sortie + 6, expert);
    sortie[8] = 0;
    sortie[9] = 3;
    eu16(sortie + 10, uint32_t(n));
    eu32(sortie + 12, uint32_t(utiles));
    for (size_t i = 0; i < n; ++i) {
        uint8_t* e = sortie + 64 + 16 * i;
        e[0] = flux[i].sorte;
        e[1] = flux[i].matrice;
        e[2] = flux[i].contexte;
        eu32(e + 4, uint32_t(dec[i]));
        eu32(e + 8, uint32_t(flux[i].octets.size()));
        eu32(e + 12, flux[i].produits);
        std::memcpy(sortie + dec[i], flux[i].octets.data(), flux[i].octets.size());
    }
    return int64_t(total);
}

bool dims_valides(const trc_dims_expert* d) {
    if (!d) return false;
    for (int j = 0; j < 3; ++j)
        if (d->lignes[j] == 0 || d->colonnes[j] == 0 || d->colonnes[j] % 32) return false;
    return true;
}

// splitmix64 (Steele, Lea, Flood 2014) and Box-Muller normals, for the synthetic generator.
struct Alea {
    uint64_t s;
    uint64_t suivant() {
        uint64_t z = (s += 0x9E3779B97F4A7C15ull);
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    double uniforme() { return double((suivant() >> 11) + 1) * (1.0 / 9007199254740993.0); }
    double normale() {
        const double u = uniforme(), v = uniforme();
        return std::sqrt(-2.0 * std::log(u)) * std::cos(6.283185307179586 * v);
    }
};

// Nearest E2M1 code of |v| (ties to the even code), sign in bit 3.
uint8_t e2m1(double v) {
    const double a = std::fabs(v);
    uint8_t c;
    if (a <= 0.25) c = 0;
    else if (a < 0.75) c = 1;
    else if (a <= 1.25) c = 2;
    else if (a < 1.75) c = 3;
    else if (a <= 2.5) c = 4;
    else if (a < 3.5) c = 5;
    else if (a <= 5.0) c = 6;
    else c = 7;
    return uint8_t(c | (std::signbit(v) ? 8 : 0));
}

float bf16_rne(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    std::memcpy(&f, &u, 4);
    return f;
}

void parallele(uint32_t n, int fils, const std::function<void(uint32_t)>& f) {
    uint32_t nf = fils > 0 ? uint32_t(fils) : std::max(1u, std::thread::hardware_concurrency());
    nf = std::min(nf, n);
    if (nf <= 1) {
        for (uint32_t i = 0; i < n; ++i) f(i);
        return;
    }
    std::vector<std::thread> t;
    std::atomic<uint32_t> suivant{0};
    for (uint32_t k = 0; k < nf; ++k)
        t.emplace_back([&] {
            for (uint32_t i; (i = suivant.fetch_add(1)) < n;) f(i);
        });
    for (auto& x : t) x.join();
}
}  // namespace

extern "C" {

int trc_table_depuis_comptes(const uint64_t* comptes, uint32_t geometrie, uint16_t* freq) {
    if (!comptes || !freq || (geometrie != 1 && geometrie != 2)) return TRC_ERR_USAGE;
    const int n = geometrie == 1 ? 256 : 16;
    std::vector<uint64_t> c(comptes, comptes + n);
    uint64_t total = 0;
    for (auto v : c) total += v;
    if (total == 0) {
        c[0] = 1;
        total = 1;
    }
    std::vector<int64_t> f(n, 0);
    for (int i = 0; i < n; ++i)
        if (c[i] > 0) f[i] = std::max<int64_t>(1, int64_t(std::round(double(c[i]) * double(M) / double(total))));
    int64_t somme = 0;
    for (auto v : f) somme += v;
    bool fait = false;
    if (geometrie == 2) {
        int imax = 0;
        for (int i = 0; i < n; ++i)
            if (f[i] >= f[imax]) imax = i;  // the last maximum
        const int64_t corrige = f[imax] + (int64_t(M) - somme);
        if (corrige >= 1) {
            f[imax] = corrige;
            fait = true;
        }
    }
    if (!fait) {
        std::vector<int> ordre(n);
        for (int i = 0; i < n; ++i) ordre[i] = i;
        std::stable_sort(ordre.begin(), ordre.end(), [&](int a, int b) { return f[a] > f[b]; });
        for (int64_t j = 0; somme != int64_t(M); ++j) {
            const int i = ordre[j % n];
            if (somme > int64_t(M) && f[i] > 1) {
                --f[i];
                --somme;
            } else if (somme < int64_t(M) && f[i] > 0) {
                ++f[i];
                ++somme;
            }
        }
    }
    for (int i = 0; i < n; ++i) freq[i] = uint16_t(f[i]);
    return TRC_OK;
}

int trc_lut_geometrie1(const uint16_t* freq, uint32_t* lut) {
    if (!freq || !lut) return TRC_ERR_USAGE;
    uint32_t somme = 0;
    for (int s = 0; s < 256; ++s) somme += freq[s];
    if (somme != M) return TRC_ERR_USAGE;
    uint32_t c = 0;
    for (uint32_t s = 0; s < 256; ++s) {
        const uint32_t f = freq[s];
        for (uint32_t i = c; i < c + f; ++i) lut[i] = s | ((f - 1) << 8) | ((i - c) << 20);
        c += f;
    }
    return TRC_OK;
}

int trc_luts_couche(const uint16_t* freqs, const uint8_t* presentes, uint32_t* luts) {
    if (!freqs || !luts) return TRC_ERR_USAGE;
    std::memset(luts, 0, sizeof(uint32_t) * 3 * 4 * M);
    for (int t = 0; t < 12; ++t) {
        if (presentes && !presentes[t]) continue;
        if (trc_lut_geometrie1(freqs + 256 * t, luts + size_t(M) * t) != TRC_OK) return TRC_ERR_USAGE;
    }
    return TRC_OK;
}

int trc_comptes_matrice(const uint8_t* blocs, uint32_t lignes, uint32_t blocs_par_ligne, int canonique, uint64_t* comptes) {
    if (!blocs || !comptes || lignes == 0 || blocs_par_ligne == 0) return TRC_ERR_USAGE;
    const Prepa p = preparer(blocs, lignes, blocs_par_ligne, canonique != 0);
    for (uint8_t d : p.delta) comptes[d] += 1;
    for (size_t n = 0; n < p.qs.size(); ++n) {
        const uint8_t k = n / 16 < p.delta.size() ? classe(p.delta[n / 16]) : 0;
        comptes[256 * (1 + k) + p.qs[n]] += 1;
    }
    return TRC_OK;
}

int64_t trc_coder_partie(const uint8_t* const* blocs, const uint8_t* const* biais, const trc_dims_expert* dims,
                         const uint16_t* freqs, int canonique, uint16_t couche, uint16_t expert, uint32_t n_delta,
                         uint32_t n_codes, uint8_t* sortie, size_t capacite, uint32_t* utiles) {
    if (!blocs || !biais || !freqs || !dims_valides(dims) || n_delta == 0 || n_codes == 0 || n_delta > 65535 ||
        n_codes > 65535)
        return -1;
    std::vector<FluxP> flux;
    for (uint32_t j = 0; j < 3; ++j) {
        const uint32_t R = dims->lignes[j], B = dims->colonnes[j] / 32;
        const Prepa p = preparer(blocs[j], R, B, canonique != 0);
        const uint16_t* td[1] = {freqs + (4 * j) * 256};
        const std::vector<uint8_t> fd = coder_g1(p.delta, n_delta, nullptr, td);
        std::vector<uint8_t> kappa(p.delta.size());
        for (size_t i = 0; i < kappa.size(); ++i) kappa[i] = classe(p.delta[i]);
        const uint16_t* tc[3] = {freqs + (4 * j + 1) * 256, freqs + (4 * j + 2) * 256, freqs + (4 * j + 3) * 256};
        const std::vector<uint8_t> fc = coder_g1(p.qs, n_codes, &kappa, tc);
        if (fd.empty() || fc.empty()) return -1;
        flux.push_back({0x01, uint8_t(j), 0xFF, R, p.med});
        flux.push_back({0x02, uint8_t(j), 0xFF, 4 * R, std::vector<uint8_t>(biais[j], biais[j] + 4ull * R)});
        flux.push_back({0x03, uint8_t(j), 0, uint32_t(p.delta.size()), fd});
        flux.push_back({0x04, uint8_t(j), 0xFF, uint32_t(p.qs.size()), fc});
    }
    return assembler(couche, expert, flux, sortie, capacite, utiles);
}

int64_t trc_coder_partie_brute(const uint8_t* const* blocs, const uint8_t* const* biais, const trc_dims_expert* dims,
                               uint16_t couche, uint16_t expert, uint8_t* sortie, size_t capacite, uint32_t* utiles) {
    if (!blocs || !biais || !dims_valides(dims)) return -1;
    std::vector<FluxP> flux;
    for (uint32_t j = 0; j < 3; ++j) {
        const uint32_t R = dims->lignes[j], B = dims->colonnes[j] / 32;
        const size_t nb = size_t(R) * B;
        std::vector<uint8_t> ech(nb), codes(16 * nb);
        for (size_t b = 0; b < nb; ++b) {
            ech[b] = blocs[j][17 * b];
            std::memcpy(&codes[16 * b], blocs[j] + 17 * b + 1, 16);
        }
        flux.push_back({0x07, uint8_t(j), 0xFF, uint32_t(nb), std::move(ech)});
        flux.push_back({0x06, uint8_t(j), 0xFF, uint32_t(16 * nb), std::move(codes)});
        flux.push_back({0x02, uint8_t(j), 0xFF, 4 * R, std::vector<uint8_t>(biais[j], biais[j] + 4ull * R)});
    }
    return assembler(couche, expert, flux, sortie, capacite, utiles);
}

int trc_synth_matrices(uint64_t graine, uint32_t lignes, uint32_t colonnes, uint32_t premier, uint32_t n,
                       uint8_t* blocs, float* biais, int fils) {
    if (!blocs || !biais || lignes == 0 || colonnes == 0 || colonnes % 32) return TRC_ERR_USAGE;
    const uint32_t B = colonnes / 32;
    parallele(n * lignes, fils, [&](uint32_t t) {
        const uint32_t x = t / lignes, r = t % lignes;
        Alea a{graine * 0x9E3779B97F4A7C15ull ^ (uint64_t(premier + x) << 32) ^ r};
        a.suivant();
        const double sigma = 0.02 * std::exp(0.3 * a.normale());
        uint8_t* ligne = blocs + (size_t(x) * lignes + r) * B * 17;
        double w[32];
        for (uint32_t b = 0; b < B; ++b) {
            double mx = 0.0;
            for (int i = 0; i < 32; ++i) {
                w[i] = sigma * a.normale();
                mx = std::max(mx, std::fabs(w[i]));
            }
            int E = mx > 0.0 ? int(std::floor(std::log2(mx))) - 2 : -127;
            E = std::min(127, std::max(-127, E));
            uint8_t* blk = ligne + 17 * b;
            blk[0] = uint8_t(E + 127);
            const double inv = std::ldexp(1.0, -E);
            for (int i = 0; i < 16; ++i) blk[1 + i] = uint8_t(e2m1(w[i] * inv) | (e2m1(w[16 + i] * inv) << 4));
        }
        biais[size_t(x) * lignes + r] = bf16_rne(float(0.01 * a.normale()));
    });
    return TRC_OK;
}

}  // extern "C"
