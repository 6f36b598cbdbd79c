// troncons_b200 — the `.trc` encoder on the GPU: geometry-1 rANS streams (rans.rs:186-228) and
// whole level-0 expert parts, byte for byte what the CPU encoders write (trc-codec rans.rs:296-334,
// lib.rs:348-428; trc-format lib.rs:882-908; the reference bench's coder_g1, banc_k.cu:277-321).
//
// Tiles are independent. One warp encodes one tile backwards (macro-steps m, sub-steps
// k = 3..0), lane l encoding byte 4 (32 m + l) + k with the table of its context: renormalise when
// x >= f << 20 (push the low 16 bits), then x = (x / f) M + (x mod f) + c. The division is a
// multiply-high and a shift (Granlund-Montgomery, "Division by invariant integers using
// multiplication", 1994, theorem 4.2 with N = 32: m = ceil(2^(32+l) / f), l = ceil(log2 f), so
// floor(x / f) = (mulhi(x, m - 2^32) + x) >> l for every x < 2^32), precomputed per symbol with
// the table in shared memory. The pushes of one sub-step go in lane order 31 .. 0 (a ballot ranks
// them) onto the tile's stack in scratch memory.
//
// A stream is then laid out by three passes: a per-stream scan of the tiles' word counts (tile
// starts, W), a per-part pass placing the streams (offsets aligned to 16, the part header and
// stream table, the streams' own headers, every gap and the tail zeroed), and a per-tile pass
// writing the tile start, the 32 final states and the stack reversed. Parts encode straight from
// the 17-byte MXFP4 blocks: a first pass takes each row's median scale and writes the row's
// deltas (lib.rs:348-373); the CODES_CTX tiles read the code bytes from the blocks, folding -0
// (v1.2), with the scale class of the block's delta as context.
#include "commun.cuh"
#include "noyaux.h"

namespace tb {

constexpr uint32_t CODEUR_WARPS = 8;
constexpr uint32_t CODEUR_TABLES_MAX = 4;
constexpr uint32_t FLUX_EXPERT = 6;    // per expert: DELTA_j, CODES_CTX_j for j = 0..2
constexpr uint32_t FLUX_PARTIE = 12;   // MEDIANES_j, BIAIS_j, DELTA_j, CODES_CTX_j
constexpr uint32_t SOURCE_OCTETS = 0;  // plain bytes, optional per-16-byte context
constexpr uint32_t SOURCE_BLOCS = 1;   // the code bytes of 17-byte MXFP4 blocks

__host__ __device__ __forceinline__ uint32_t classe_delta(uint32_t d) { return d < 128u ? 0u : (d == 128u ? 1u : 2u); }
__device__ __forceinline__ uint32_t canonique4(uint32_t o) {  // nibble 8 (-0) -> 0, in each byte of a word
    const uint32_t lo = o & 0x0F0F0F0Fu, hi = (o >> 4) & 0x0F0F0F0Fu;
    const uint32_t lo8 = lo & ~(lo << 1) & ~(lo << 2) & ~(lo << 3) & 0x08080808u;  // nibble == 8
    const uint32_t hi8 = hi & ~(hi << 1) & ~(hi << 2) & ~(hi << 3) & 0x08080808u;
    return ((lo ^ lo8) | ((hi ^ hi8) << 4));
}

// One stream of every expert of a call.
struct FluxCodage {
    const uint8_t* src;    // SOURCE_OCTETS: the bytes (expert e's at src + e * src_pas)
    const uint8_t* kappa;  // per-16-byte context bytes (expert e's at kappa + e * kappa_pas), or null
    const uint16_t* freqs; // n_tables tables u16[256]
    uint64_t src_pas, kappa_pas;
    uint32_t source, matrice, nb, canonique;  // SOURCE_BLOCS: matrix j of the descriptors, R*B blocks
    uint32_t n_kappa, kappa_classe;           // kappa_classe: context = scale class of the byte
    uint32_t n_tables, P, N, T;
    uint32_t bloc0, tuile0;  // first CTA and first tile of this stream within an expert's
    uint64_t pile0;          // first stack word of this stream within an expert's
};

struct PlanCodage {
    FluxCodage f[FLUX_EXPERT];
    const DescCodage* descs;  // parts (device), or null for one stream
    uint32_t n_flux, n_exp, blocs_exp, tuiles_exp, tuiles_bloc, erreur_pas;
    uint64_t mots_exp;
    uint16_t* piles;
    uint32_t *n_mots, *debuts, *etats, *W, *erreur;
};

// Stream s of the plan for CTA or tile index i within an expert (by their first indices).
__device__ __forceinline__ uint32_t flux_du_bloc(const PlanCodage& p, uint32_t b) {
    uint32_t s = 0;
    while (s + 1 < p.n_flux && b >= p.f[s + 1].bloc0) ++s;
    return s;
}
__device__ __forceinline__ uint32_t flux_de_tuile(const PlanCodage& p, uint32_t g) {
    uint32_t s = 0;
    while (s + 1 < p.n_flux && g >= p.f[s + 1].tuile0) ++s;
    return s;
}

// ---------------------------------------------------------------- tiles

__global__ void __launch_bounds__(CODEUR_WARPS * 32) k_coder_tuiles(const __grid_constant__ PlanCodage p) {
    __shared__ uint2 S[CODEUR_TABLES_MAX][256];  // x: f | c << 13 | l << 25; y: m - 2^32
    attendre_amont();
    liberer_aval();
    const uint32_t e = blockIdx.x / p.blocs_exp, bl = blockIdx.x % p.blocs_exp;
    const FluxCodage& f = p.f[flux_du_bloc(p, bl)];
    const uint32_t voie = threadIdx.x & 31u, w = threadIdx.x >> 5;
    if (w < f.n_tables) {  // table w: lane l holds symbols 8l .. 8l + 7; a warp scan gives the starts
        uint32_t fr[8], somme = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            fr[i] = f.freqs[256u * w + 8u * voie + i];
            somme += fr[i];
        }
        uint32_t incl = somme;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
            if (voie >= uint32_t(d)) incl += v;
        }
        uint32_t c = incl - somme;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t fi = fr[i] > 4096u ? 0u : fr[i];
            const uint32_t l = fi <= 1u ? 0u : 32u - __clz(fi - 1u);
            const uint64_t m = fi == 0u ? (1ull << 32) : ((1ull << (32 + l)) + fi - 1u) / fi;
            S[w][8u * voie + i] = make_uint2(fi | ((c & 0xFFFu) << 13) | (l << 25), uint32_t(m - (1ull << 32)));
            c += fr[i];
        }
    }
    __syncthreads();
    // The stream's fields in registers: the stack stores below could alias the plan's memory for
    // the compiler, which would then reload them from it at every macro-step.
    const uint32_t source = f.source, nb = f.nb, canonique = f.canonique, n_kappa = f.n_kappa;
    const uint32_t kappa_classe = f.kappa_classe, n_tables = f.n_tables, N = f.N, T = f.T;
    const uint32_t n_macro = f.P / 128u;
    const uint8_t* src = source == SOURCE_OCTETS ? f.src + e * f.src_pas
                                                 : reinterpret_cast<const uint8_t*>(p.descs[e].blocs[f.matrice]);
    const uint8_t* kappa = f.kappa != nullptr ? f.kappa + e * f.kappa_pas : nullptr;
    uint16_t* const piles = p.piles + uint64_t(e) * p.mots_exp + f.pile0;
    const uint64_t g0 = uint64_t(e) * p.tuiles_exp + f.tuile0;
    const uint32_t dessus = voie == 31u ? 0u : (0xFFFFFFFFu << (voie + 1u));  // lanes above this one
    uint32_t manque = 0;
    const uint32_t t_debut = (bl - f.bloc0) * p.tuiles_bloc;
    const uint32_t t_fin = min(t_debut + p.tuiles_bloc, T);
    // The word of lane `voie` at macro-step m and its context.
    auto charger = [&](uint32_t m, uint32_t& mot, uint32_t& ctx) {
        const uint32_t wi = m * 32u + voie, b = wi >> 2;
        if (source == SOURCE_OCTETS) {
            mot = __ldg(reinterpret_cast<const uint32_t*>(src) + wi);
        } else if (b < nb) {
            const uint8_t* q = src + 17ull * b + 1u + 4u * (wi & 3u);
            mot = uint32_t(__ldg(q)) | (uint32_t(__ldg(q + 1)) << 8) | (uint32_t(__ldg(q + 2)) << 16) |
                  (uint32_t(__ldg(q + 3)) << 24);
            if (canonique) mot = canonique4(mot);
        } else {
            mot = 0;
        }
        ctx = 0;
        if (kappa != nullptr && b < n_kappa) {
            ctx = __ldg(kappa + b);
            if (kappa_classe) ctx = classe_delta(ctx);
        }
    };
    constexpr int AVANCE = 4;  // macro-steps loaded ahead of the one being encoded
    for (uint32_t t = t_debut + w; t < t_fin; t += CODEUR_WARPS) {
        const uint32_t m0 = t * N, m1 = min(m0 + N, n_macro);
        uint16_t* pile = piles + uint64_t(t) * 128u * N;
        uint32_t x = L, np = 0;
        uint32_t mw[AVANCE], cw[AVANCE];
#pragma unroll
        for (int i = 0; i < AVANCE; ++i) {
            mw[i] = cw[i] = 0;
            if (m1 > m0 + uint32_t(i)) charger(m1 - 1u - uint32_t(i), mw[i], cw[i]);
        }
        for (uint32_t m = m1; m-- > m0;) {
            const uint32_t mot_c = mw[0], ctx_c = cw[0] < n_tables ? cw[0] : 0u;
            manque |= cw[0] >= n_tables ? 1u : 0u;  // a context without a table: an encoding error
#pragma unroll
            for (int i = 0; i + 1 < AVANCE; ++i) {
                mw[i] = mw[i + 1];
                cw[i] = cw[i + 1];
            }
            if (m >= m0 + uint32_t(AVANCE)) charger(m - uint32_t(AVANCE), mw[AVANCE - 1], cw[AVANCE - 1]);
#pragma unroll
            for (int k = 3; k >= 0; --k) {
                const uint2 ent = S[ctx_c][(mot_c >> (8 * k)) & 0xFFu];
                const uint32_t fr = ent.x & 0x1FFFu, c = (ent.x >> 13) & 0xFFFu, l = ent.x >> 25;
                manque |= fr == 0u ? 1u : 0u;
                const bool pousse = (x >> 20) >= fr;
                const uint32_t vote = __ballot_sync(0xFFFFFFFFu, pousse);
                if (pousse) pile[np + __popc(vote & dessus)] = uint16_t(x & 0xFFFFu);
                np += __popc(vote);
                const uint32_t xv = pousse ? x >> 16 : x;
                const uint32_t q = uint32_t((uint64_t(__umulhi(xv, ent.y)) + xv) >> l);
                x = (q << 12) + (xv - q * fr) + c;
            }
        }
        p.etats[(g0 + t) * 32u + voie] = x;
        if (voie == 0) p.n_mots[g0 + t] = np;
    }
    if (__any_sync(0xFFFFFFFFu, manque) && voie == 0) atomicOr(p.erreur + e * p.erreur_pas, 1u);
}

// ---------------------------------------------------------------- layout

// One block per (stream, expert): tile starts (exclusive prefix sum of the word counts, in
// tile order) and the stream's word count W.
__global__ void __launch_bounds__(1024) k_flux_scan(const __grid_constant__ PlanCodage p) {
    __shared__ uint32_t part[1024];
    __shared__ uint32_t base;
    attendre_amont();
    liberer_aval();
    const FluxCodage& f = p.f[blockIdx.x];
    const uint32_t e = blockIdx.y;
    const uint64_t g0 = uint64_t(e) * p.tuiles_exp + f.tuile0;
    if (threadIdx.x == 0) base = 0;
    __syncthreads();
    for (uint32_t t0 = 0; t0 < f.T; t0 += 1024u) {
        const uint32_t t = t0 + threadIdx.x;
        const uint32_t v = t < f.T ? p.n_mots[g0 + t] : 0u;
        part[threadIdx.x] = v;
        __syncthreads();
        for (uint32_t d = 1; d < 1024u; d <<= 1) {
            const uint32_t a = threadIdx.x >= d ? part[threadIdx.x - d] : 0u;
            __syncthreads();
            part[threadIdx.x] += a;
            __syncthreads();
        }
        if (t < f.T) p.debuts[g0 + t] = base + part[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == 1023u) base += part[1023];
        __syncthreads();
    }
    if (threadIdx.x == 0) p.W[e * p.n_flux + blockIdx.x] = base;
}

__host__ __device__ __forceinline__ uint64_t longueur_flux(uint32_t T, uint32_t W) {
    return (16ull + 132ull * T + 2ull * W + 15ull) & ~15ull;
}

// The stream's own 16-byte header and its zero padding, by one warp.
__device__ __forceinline__ void tete_flux(uint8_t* d, const FluxCodage& f, uint32_t W, uint32_t voie) {
    if (voie == 0) {
        uint32_t* h = reinterpret_cast<uint32_t*>(d);
        h[0] = f.P;
        h[1] = (f.N & 0xFFFFu) | (1u << 16);  // N, geometry 1, reserved 0
        h[2] = f.T;
        h[3] = W;
    }
    const uint64_t fin = 16ull + 132ull * f.T + 2ull * W;
    for (uint64_t o = fin + voie; o < longueur_flux(f.T, W); o += 32u) d[o] = 0;
}

// Offsets of a part's 12 streams, its useful and total lengths (lib.rs:882-908).
struct PlacePartie {
    uint64_t dec[FLUX_PARTIE], lg[FLUX_PARTIE], utiles, total;
};

__device__ __forceinline__ void placer(const PlanCodage& p, uint32_t e, const Dims& dims, PlacePartie& pl) {
    uint64_t o = 64u + 16u * FLUX_PARTIE;
    for (uint32_t i = 0; i < FLUX_PARTIE; ++i) {
        const uint32_t j = i / 4u, sorte = i % 4u, R = dims.lignes[j];
        const uint32_t s = 2u * j + (sorte == 3u ? 1u : 0u);
        const uint64_t lg = sorte == 0u ? R : sorte == 1u ? 4ull * R : longueur_flux(p.f[s].T, p.W[e * p.n_flux + s]);
        o = (o + 15u) & ~uint64_t(15);
        pl.dec[i] = o;
        pl.lg[i] = lg;
        o += lg;
    }
    pl.utiles = o;
    pl.total = (o + 4095u) & ~uint64_t(4095);
}

__device__ __forceinline__ void eu32(uint8_t* d, uint32_t v) {
    d[0] = uint8_t(v);
    d[1] = uint8_t(v >> 8);
    d[2] = uint8_t(v >> 16);
    d[3] = uint8_t(v >> 24);
}

// One warp per part (or for the lone stream): placement, header, stream table, the streams'
// headers, every gap and the tail zeroed; octets[2e] = total length (0 on an encoding error),
// octets[2e + 1] = useful bytes. Nothing is written when the part does not fit its capacity.
__global__ void __launch_bounds__(32) k_parties_tete(const __grid_constant__ PlanCodage p, Dims dims,
                                                     uint32_t couche, uint8_t* sortie_seule, uint64_t capacite_seule,
                                                     uint64_t* octets) {
    attendre_amont();
    liberer_aval();
    const uint32_t e = blockIdx.x, voie = threadIdx.x;
    const bool erreur = p.erreur[e * p.erreur_pas] != 0u;
    if (p.descs == nullptr) {  // one stream, written at sortie_seule
        const uint32_t W = p.W[0];
        const uint64_t lg = longueur_flux(p.f[0].T, W);
        if (voie == 0) octets[0] = erreur ? 0ull : lg;
        if (!erreur && lg <= capacite_seule) tete_flux(sortie_seule, p.f[0], W, voie);
        return;
    }
    PlacePartie pl;
    placer(p, e, dims, pl);
    if (voie == 0) {
        octets[2u * e] = erreur ? 0ull : pl.total;
        octets[2u * e + 1u] = pl.utiles;
    }
    const DescCodage& d = p.descs[e];
    if (erreur || pl.total > d.capacite) return;
    uint8_t* s = reinterpret_cast<uint8_t*>(d.sortie);
    for (uint32_t o = voie; o < 64u + 16u * FLUX_PARTIE; o += 32u) s[o] = 0;
    __syncwarp();
    if (voie == 0) {
        eu32(s, 0x30435254u);  // "TRC0"
        s[4] = uint8_t(couche);
        s[5] = uint8_t(couche >> 8);
        s[6] = uint8_t(d.expert);
        s[7] = uint8_t(d.expert >> 8);
        s[8] = 0;  // level 0
        s[9] = 3;  // matrices
        s[10] = uint8_t(FLUX_PARTIE);
        s[11] = 0;
        eu32(s + 12, uint32_t(pl.utiles));
    }
    if (voie < FLUX_PARTIE) {
        const uint32_t i = voie, j = i / 4u, sorte = i % 4u;
        uint8_t* t = s + 64u + 16u * i;
        t[0] = uint8_t(sorte + 1u);  // MEDIANES 0x01, BIAIS 0x02, DELTA 0x03, CODES_CTX 0x04
        t[1] = uint8_t(j);
        t[2] = sorte == 2u ? 0u : 0xFFu;
        eu32(t + 4, uint32_t(pl.dec[i]));
        eu32(t + 8, uint32_t(pl.lg[i]));
        const uint32_t R = dims.lignes[j];
        const uint32_t produits = sorte == 0u ? R : sorte == 1u ? 4u * R : p.f[2u * j + (sorte == 3u ? 1u : 0u)].P;
        eu32(t + 12, produits);
    }
    // gaps before each stream, and the tail
    for (uint32_t i = 0; i < FLUX_PARTIE; ++i) {
        const uint64_t avant = i == 0 ? 64u + 16u * FLUX_PARTIE : pl.dec[i - 1] + pl.lg[i - 1];
        for (uint64_t o = avant + voie; o < pl.dec[i]; o += 32u) s[o] = 0;
    }
    for (uint64_t o = pl.utiles + voie; o < pl.total; o += 32u) s[o] = 0;
    for (uint32_t j = 0; j < 3; ++j)
        for (uint32_t c = 0; c < 2; ++c) {
            const uint32_t sf = 2u * j + c;
            tete_flux(s + pl.dec[4u * j + 2u + c], p.f[sf], p.W[e * p.n_flux + sf], voie);
        }
}

// Per tile: its start, its 32 final states and its words (the stack reversed). Parts: the CTAs
// after the tiles copy the medians and the biases.
__global__ void __launch_bounds__(256) k_parties_corps(const __grid_constant__ PlanCodage p, Dims dims,
                                                       const uint8_t* __restrict__ medianes, uint64_t med_pas,
                                                       uint8_t* sortie_seule, uint64_t capacite_seule,
                                                       const uint64_t* octets) {
    attendre_amont();
    liberer_aval();
    const uint32_t e = blockIdx.y, g = blockIdx.x;
    uint8_t* s;
    uint64_t dec_flux[FLUX_EXPERT];
    if (p.descs == nullptr) {
        if (octets[0] == 0 || octets[0] > capacite_seule) return;
        s = sortie_seule;
        dec_flux[0] = 0;
    } else {
        const DescCodage& d = p.descs[e];
        if (octets[2u * e] == 0 || octets[2u * e] > d.capacite) return;
        s = reinterpret_cast<uint8_t*>(d.sortie);
        PlacePartie pl;
        placer(p, e, dims, pl);
        if (g >= p.tuiles_exp) {  // medians and biases of matrix j
            const uint32_t c = g - p.tuiles_exp, j = c / 2u, R = dims.lignes[j];
            if (c % 2u == 0) {
                const uint8_t* m = medianes + e * med_pas;
                uint64_t mo = 0;
                for (uint32_t a = 0; a < j; ++a) mo += al256(dims.lignes[a]);
                for (uint32_t o = threadIdx.x; o < R; o += blockDim.x) s[pl.dec[4u * j] + o] = m[mo + o];
            } else {
                const uint32_t* b = reinterpret_cast<const uint32_t*>(d.biais[j]);
                uint32_t* o32 = reinterpret_cast<uint32_t*>(s + pl.dec[4u * j + 1u]);
                for (uint32_t o = threadIdx.x; o < R; o += blockDim.x) o32[o] = b[o];
            }
            return;
        }
        for (uint32_t i = 0; i < FLUX_EXPERT; ++i) dec_flux[i] = pl.dec[4u * (i / 2u) + 2u + i % 2u];
    }
    const uint32_t sf = flux_de_tuile(p, g);
    const FluxCodage& f = p.f[sf];
    const uint32_t t = g - f.tuile0;
    const uint64_t gi = uint64_t(e) * p.tuiles_exp + g;
    uint8_t* d = s + dec_flux[sf];
    const uint32_t debut = p.debuts[gi], n = p.n_mots[gi];
    if (threadIdx.x == 0) reinterpret_cast<uint32_t*>(d + 16)[t] = debut;
    if (threadIdx.x < 32u) reinterpret_cast<uint32_t*>(d + 16 + 4ull * f.T)[32u * t + threadIdx.x] = p.etats[gi * 32u + threadIdx.x];
    uint16_t* mots = reinterpret_cast<uint16_t*>(d + 16 + 132ull * f.T) + debut;
    const uint16_t* pile = p.piles + uint64_t(e) * p.mots_exp + f.pile0 + uint64_t(t) * 128u * f.N;
    for (uint32_t j = threadIdx.x; j < n; j += blockDim.x) mots[j] = pile[n - 1u - j];
}

// ---------------------------------------------------------------- rows: medians, deltas, counts

// One warp per row (grid-stride over the rows of every matrix of every expert): the row's median
// scale (tri[B/2] of its sorted scales, by a 256-bin count) and its deltas (e - med + 128), into
// scratch; the last row of a matrix zeroes the deltas' padding. With `comptes` (u64[3][4][256],
// accumulated): the layer's symbol counts instead (lib.rs:393-401): DELTA, and each code byte
// under the class of its block's delta, padding included.
__global__ void __launch_bounds__(256) k_lignes(const DescCodage* __restrict__ descs, uint32_t n_exp,
                                                Dims dims, uint32_t canonique, uint8_t* medianes,
                                                uint64_t med_pas, uint8_t* deltas, uint64_t delta_pas,
                                                unsigned long long* comptes) {
    __shared__ uint32_t H[CODEUR_WARPS][256];
    __shared__ uint32_t C[3][4][256];
    attendre_amont();
    liberer_aval();
    const uint32_t voie = threadIdx.x & 31u, w = threadIdx.x >> 5;
    if (comptes != nullptr)
        for (uint32_t i = threadIdx.x; i < 3u * 4u * 256u; i += blockDim.x) (&C[0][0][0])[i] = 0;
    __syncthreads();
    const uint64_t lignes_exp = uint64_t(dims.lignes[0]) + dims.lignes[1] + dims.lignes[2];
    const uint64_t n_lignes = lignes_exp * n_exp;
    for (uint64_t li = uint64_t(blockIdx.x) * CODEUR_WARPS + w; li < n_lignes; li += uint64_t(gridDim.x) * CODEUR_WARPS) {
        const uint32_t e = uint32_t(li / lignes_exp);
        uint32_t r = uint32_t(li % lignes_exp), j = 0;
        while (r >= dims.lignes[j]) r -= dims.lignes[j++];
        const uint32_t B = dims.colonnes[j] / 32u, R = dims.lignes[j];
        const uint8_t* ligne = reinterpret_cast<const uint8_t*>(descs[e].blocs[j]) + 17ull * B * r;
        for (uint32_t i = voie; i < 256u; i += 32u) H[w][i] = 0;
        __syncwarp();
        for (uint32_t b = voie; b < B; b += 32u) atomicAdd(&H[w][__ldg(ligne + 17ull * b)], 1u);
        __syncwarp();
        // the smallest value v with count(<= v) > B / 2: lane l sums bins 8l .. 8l + 7
        uint32_t h[8], somme = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            h[i] = H[w][8u * voie + i];
            somme += h[i];
        }
        uint32_t incl = somme;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
            if (voie >= uint32_t(d)) incl += v;
        }
        const uint32_t rang = B / 2u;
        uint32_t med = 0;
        const uint32_t ici = __ballot_sync(0xFFFFFFFFu, incl > rang && incl - somme <= rang);
        const uint32_t l0 = __ffs(ici) - 1u;
        if (voie == l0) {
            uint32_t c = incl - somme;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                c += h[i];
                if (c > rang) {
                    med = 8u * voie + i;
                    break;
                }
            }
        }
        med = __shfl_sync(0xFFFFFFFFu, med, l0);
        __syncwarp();
        uint64_t mo = 0, dof = 0;
        for (uint32_t a = 0; a < j; ++a) {
            mo += al256(dims.lignes[a]);
            dof += al256((uint64_t(dims.lignes[a]) * (dims.colonnes[a] / 32u) + 127u) / 128u * 128u);
        }
        if (comptes == nullptr) {
            if (voie == 0) medianes[e * med_pas + mo + r] = uint8_t(med);
            uint8_t* dl = deltas + e * delta_pas + dof;
            for (uint32_t b = voie; b < B; b += 32u) dl[uint64_t(r) * B + b] = uint8_t(__ldg(ligne + 17ull * b) - med + 128u);
            if (r == R - 1u) {
                const uint64_t nb = uint64_t(R) * B, pd = (nb + 127u) / 128u * 128u;
                for (uint64_t o = nb + voie; o < pd; o += 32u) dl[o] = 0;
            }
        } else {
            for (uint32_t o = voie; o < 17u * B; o += 32u) {
                const uint32_t b = o / 17u, k = o - 17u * b;
                const uint32_t delta = (__ldg(ligne + 17ull * b) - med + 128u) & 0xFFu;
                if (k == 0) {
                    atomicAdd(&C[j][0][delta], 1u);
                } else {
                    uint32_t q = __ldg(ligne + o);
                    if (canonique) q = canonique4(q) & 0xFFu;
                    atomicAdd(&C[j][1u + classe_delta(delta)][q], 1u);
                }
            }
        }
    }
    if (comptes == nullptr) return;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < 3u * 4u * 256u; i += blockDim.x) {
        uint32_t v = (&C[0][0][0])[i];
        if (blockIdx.x == 0 && i % 1024u == 0u) {  // padding: delta 0 (table DELTA), code 0 (class 0)
            const uint32_t j = i / 1024u;
            const uint64_t nb = uint64_t(dims.lignes[j]) * (dims.colonnes[j] / 32u);
            atomicAdd(comptes + i, (unsigned long long)((nb + 127u) / 128u * 128u - nb) * n_exp);
        }
        if (blockIdx.x == 0 && i % 1024u == 256u) {
            const uint32_t j = i / 1024u;
            const uint64_t nb = uint64_t(dims.lignes[j]) * (dims.colonnes[j] / 32u);
            atomicAdd(comptes + i, (unsigned long long)((16u * nb + 127u) / 128u * 128u - 16u * nb) * n_exp);
        }
        if (v != 0) atomicAdd(comptes + i, (unsigned long long)v);
    }
}

// ---------------------------------------------------------------- plans and launches

namespace {

uint32_t tuiles_par_bloc(uint32_t N) { return CODEUR_WARPS * std::max(1u, std::min(16u, 64u / N)); }

// Places stream f after the plan's current streams (CTAs, tiles, stack words).
void ajouter_flux(PlanCodage& p, FluxCodage f) {
    f.T = (f.P / 128u + f.N - 1u) / f.N;
    f.bloc0 = p.blocs_exp;
    f.tuile0 = p.tuiles_exp;
    f.pile0 = p.mots_exp;
    p.blocs_exp += (f.T + p.tuiles_bloc - 1u) / p.tuiles_bloc;
    p.tuiles_exp += f.T;
    p.mots_exp += uint64_t(f.T) * 128u * f.N;
    p.f[p.n_flux++] = f;
}

// Scratch of a plan: per expert its stacks, word counts, tile starts, states, W and error flag.
struct EspaceCodage {
    uint64_t piles, n_mots, debuts, etats, W, erreur, med, deltas, total;
};

EspaceCodage espace_codage(const PlanCodage& p, uint64_t med_exp, uint64_t deltas_exp) {
    EspaceCodage z{};
    const uint64_t n = p.n_exp;
    uint64_t o = 0;
    z.piles = o;
    o += al256(n * p.mots_exp * 2u);
    z.n_mots = o;
    o += al256(n * p.tuiles_exp * 4u);
    z.debuts = o;
    o += al256(n * p.tuiles_exp * 4u);
    z.etats = o;
    o += al256(n * p.tuiles_exp * 128u);
    z.W = o;
    o += al256(n * FLUX_EXPERT * 4u);
    z.erreur = o;
    o += al256(n * 4u);
    z.med = o;
    o += n * med_exp;
    z.deltas = o;
    o += n * deltas_exp;
    z.total = o;
    return z;
}

void brancher(PlanCodage& p, const EspaceCodage& z, uint8_t* espace) {
    p.piles = reinterpret_cast<uint16_t*>(espace + z.piles);
    p.n_mots = reinterpret_cast<uint32_t*>(espace + z.n_mots);
    p.debuts = reinterpret_cast<uint32_t*>(espace + z.debuts);
    p.etats = reinterpret_cast<uint32_t*>(espace + z.etats);
    p.W = reinterpret_cast<uint32_t*>(espace + z.W);
    p.erreur = reinterpret_cast<uint32_t*>(espace + z.erreur);
    p.erreur_pas = 1;
}

PlanCodage plan_flux(uint32_t P, uint32_t N) {
    PlanCodage p{};
    p.n_exp = 1;
    p.tuiles_bloc = tuiles_par_bloc(N);
    FluxCodage f{};
    f.P = P;
    f.N = N;
    ajouter_flux(p, f);
    return p;
}

uint64_t med_expert(const Dims& d) { return al256(d.lignes[0]) + al256(d.lignes[1]) + al256(d.lignes[2]); }
uint64_t deltas_expert(const Dims& d) {
    uint64_t o = 0;
    for (int j = 0; j < 3; ++j) o += al256((uint64_t(d.lignes[j]) * (d.colonnes[j] / 32u) + 127u) / 128u * 128u);
    return o;
}

PlanCodage plan_parties(const Dims& d, uint32_t n, uint32_t n_delta, uint32_t n_codes) {
    PlanCodage p{};
    p.n_exp = n;
    p.tuiles_bloc = tuiles_par_bloc(std::min(n_delta, n_codes));
    for (uint32_t j = 0; j < 3; ++j) {
        const uint32_t nb = d.lignes[j] * (d.colonnes[j] / 32u);
        FluxCodage fd{}, fc{};
        fd.source = SOURCE_OCTETS;
        fd.P = (nb + 127u) / 128u * 128u;
        fd.N = n_delta;
        fd.n_tables = 1;
        ajouter_flux(p, fd);
        fc.source = SOURCE_BLOCS;
        fc.matrice = j;
        fc.nb = nb;
        fc.P = (16u * nb + 127u) / 128u * 128u;
        fc.N = n_codes;
        fc.n_tables = 3;
        fc.kappa_classe = 1;
        fc.n_kappa = fd.P;
        ajouter_flux(p, fc);
    }
    return p;
}

}  // namespace

uint64_t coder_flux_espace(uint32_t P, uint32_t N) {
    return espace_codage(plan_flux(P, N), 0, 0).total;
}

cudaError_t lancer_coder_flux(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, uint32_t n_kappa,
                              const uint16_t* freqs, uint32_t n_tables, uint8_t* sortie, uint64_t capacite, uint64_t* octets,
                              uint8_t* espace, cudaStream_t flux) {
    PlanCodage p = plan_flux(P, N);
    p.f[0].src = src;
    p.f[0].kappa = kappa;
    p.f[0].n_kappa = kappa != nullptr ? n_kappa : 0u;
    p.f[0].freqs = freqs;
    p.f[0].n_tables = n_tables;
    const EspaceCodage z = espace_codage(p, 0, 0);
    brancher(p, z, espace);
    cudaError_t e = cudaMemsetAsync(p.erreur, 0, 4, flux);
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_coder_tuiles, dim3(p.blocs_exp), dim3(CODEUR_WARPS * 32), 0, flux, p);
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_flux_scan, dim3(1, 1), dim3(1024), 0, flux, p);
    if (e != cudaSuccess) return e;
    const Dims dims{};
    e = lancer_pdl(k_parties_tete, dim3(1), dim3(32), 0, flux, p, dims, 0u, sortie, capacite, octets);
    if (e != cudaSuccess) return e;
    return lancer_pdl(k_parties_corps, dim3(p.tuiles_exp, 1), dim3(256), 0, flux, p, dims,
                      static_cast<const uint8_t*>(nullptr), uint64_t(0), sortie, capacite, static_cast<const uint64_t*>(octets));
}

uint64_t coder_parties_espace(const Dims& dims, uint32_t n, uint32_t n_delta, uint32_t n_codes) {
    return espace_codage(plan_parties(dims, n, n_delta, n_codes), med_expert(dims), deltas_expert(dims)).total;
}

cudaError_t lancer_coder_parties(const DescCodage* descs, uint32_t n, const Dims& dims, const uint16_t* freqs,
                                 bool canonique, uint16_t couche, uint32_t n_delta, uint32_t n_codes, uint64_t* octets,
                                 uint8_t* espace, int sms, cudaStream_t flux) {
    PlanCodage p = plan_parties(dims, n, n_delta, n_codes);
    const uint64_t med_pas = med_expert(dims), delta_pas = deltas_expert(dims);
    const EspaceCodage z = espace_codage(p, med_pas, delta_pas);
    brancher(p, z, espace);
    p.descs = descs;
    uint64_t dof = 0;
    for (uint32_t j = 0; j < 3; ++j) {
        FluxCodage& fd = p.f[2u * j];
        FluxCodage& fc = p.f[2u * j + 1u];
        fd.src = espace + z.deltas + dof;
        fd.src_pas = delta_pas;
        fd.freqs = freqs + 256u * (4u * j);
        fc.kappa = espace + z.deltas + dof;
        fc.kappa_pas = delta_pas;
        fc.freqs = freqs + 256u * (4u * j + 1u);
        fc.canonique = canonique ? 1u : 0u;
        dof += al256(fd.P);
    }
    cudaError_t e = cudaMemsetAsync(p.erreur, 0, 4ull * n, flux);
    if (e != cudaSuccess) return e;
    const uint64_t lignes = (uint64_t(dims.lignes[0]) + dims.lignes[1] + dims.lignes[2]) * n;
    const uint32_t blocs_lignes = uint32_t(std::min<uint64_t>((lignes + CODEUR_WARPS - 1) / CODEUR_WARPS, uint64_t(sms) * 8u));
    e = lancer_pdl(k_lignes, dim3(blocs_lignes), dim3(256), 0, flux, descs, n, dims, canonique ? 1u : 0u, espace + z.med,
                   med_pas, espace + z.deltas, delta_pas, static_cast<unsigned long long*>(nullptr));
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_coder_tuiles, dim3(p.blocs_exp * n), dim3(CODEUR_WARPS * 32), 0, flux, p);
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_flux_scan, dim3(FLUX_EXPERT, n), dim3(1024), 0, flux, p);
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_parties_tete, dim3(n), dim3(32), 0, flux, p, dims, uint32_t(couche), static_cast<uint8_t*>(nullptr),
                   uint64_t(0), octets);
    if (e != cudaSuccess) return e;
    return lancer_pdl(k_parties_corps, dim3(p.tuiles_exp + 6u, n), dim3(256), 0, flux, p, dims,
                      static_cast<const uint8_t*>(espace + z.med), med_pas, static_cast<uint8_t*>(nullptr), uint64_t(0),
                      static_cast<const uint64_t*>(octets));
}

cudaError_t lancer_comptes(const DescCodage* descs, uint32_t n, const Dims& dims, bool canonique,
                           uint64_t* comptes, int sms, cudaStream_t flux) {
    const uint64_t lignes = (uint64_t(dims.lignes[0]) + dims.lignes[1] + dims.lignes[2]) * n;
    const uint32_t blocs = uint32_t(std::min<uint64_t>((lignes + CODEUR_WARPS - 1) / CODEUR_WARPS, uint64_t(sms) * 4u));
    return lancer_pdl(k_lignes, dim3(blocs), dim3(256), 0, flux, descs, n, dims, canonique ? 1u : 0u,
                      static_cast<uint8_t*>(nullptr), uint64_t(0), static_cast<uint8_t*>(nullptr), uint64_t(0),
                      reinterpret_cast<unsigned long long*>(comptes));
}

}  // namespace tb
