// troncons_b200 — device definitions shared by every kernel: the `.trc` part and rANS stream
// layouts, the SoA slot layout, and the warp-level interleaved rANS decoder.
//
// Formats (read, never changed): part = 64-byte header + 16-byte stream descriptors + streams
// aligned to 16 (trc-format/src/lib.rs:779-908; ARCHITECTURE.md 4.8); rANS stream = 16-byte
// header, tile starts u32[T], lane states u32[32T], words u16[W] (rans.rs:169-280, 4.9.1).
//
// Decoding (rans.rs:388-451, the normative form): one warp decodes one tile, lane l holding
// the rANS state of lane l. Per sub-step every lane looks its state up in the LUT, and lanes
// whose state drops under L pull a 16-bit word, lanes in increasing order, from the tile's
// shared word stream: the word position is the tile pointer plus the number of lower lanes
// that also pull (ballot + popc). B200 specifics:
//   - the tile's words are staged in a per-warp shared-memory ring by asynchronous 16-byte
//     copies (cp.async, zero-filled past the tile's end) issued three 512-byte chunks ahead;
//   - every lane pre-loads the ring word at (pointer + lane) while its LUT entry is in flight,
//     so a renormalisation costs one shuffle on the dependent chain;
//   - the LUTs live in shared memory; the output byte is inserted with one byte permute;
//   - the kernels software-pipeline their per-macro-step consumer (scales, GEMV) one macro-step
//     behind the decode, branch-free, so it overlaps the decode chain's latency.
// No floating-point atomics; integer counters only (the determinism rule of commun.cuh:11-12).
#pragma once

#include <cstdint>
#include <type_traits>

namespace tb {

template <int K>
using Etape = std::integral_constant<int, K>;

constexpr uint32_t M = 4096u;     // 12-bit probabilities
constexpr uint32_t L = 65536u;    // lower bound of the state
constexpr uint32_t VOIES = 32u;   // lanes per tile
constexpr uint32_t MAGIE_PARTIE0 = 0x30435254u;  // "TRC0"

constexpr uint8_t SORTE_MEDIANES = 0x01;
constexpr uint8_t SORTE_BIAIS = 0x02;
constexpr uint8_t SORTE_DELTA = 0x03;
constexpr uint8_t SORTE_CODES_CTX = 0x04;
constexpr uint8_t SORTE_CODES_BRUTS = 0x06;
constexpr uint8_t SORTE_ECHELLES_BRUTES = 0x07;

constexpr int CTL_HORS_L = 0;
constexpr int CTL_FORMAT = 1;
constexpr int CTL_POINTEUR = 2;
constexpr int CTL_ATTENTE = 3;  // a bounded wait between two warps of a block gave up (never expected)

// Per-warp word ring: 1024 words (2 KiB) refilled by chunks of 256 words (32 lanes x 16 B),
// followed by a 64-word mirror of its first 64 words so that ring index + lane never wraps.
constexpr uint32_t ANNEAU_MOTS = 1024u;
constexpr uint32_t MIROIR_MOTS = 64u;
constexpr uint32_t ANNEAU_ALLOC = ANNEAU_MOTS + MIROIR_MOTS;  // words allocated per warp
constexpr uint32_t TRANCHE_MOTS = 256u;

struct Dims {
    uint32_t lignes[3];
    uint32_t colonnes[3];
};

__host__ __device__ __forceinline__ uint64_t al256(uint64_t x) { return (x + 255u) & ~uint64_t(255); }

// SoA slot layout of one matrix (abi.rs:69-89): codes at 0, scales at al256(16 nb), biases at
// al256(scales + nb), stride al256(biases + 4R). `base` = offset of the matrix in the slot.
struct Disposition {
    uint64_t base, echelles, biais, pas;
};

__host__ __device__ inline Disposition disposition_matrice(uint32_t R, uint32_t C) {
    const uint64_t nb = uint64_t(R) * (C / 32u);
    Disposition d;
    d.base = 0;
    d.echelles = al256(nb * 16u);
    d.biais = al256(d.echelles + nb);
    d.pas = al256(d.biais + 4ull * R);
    return d;
}

__host__ __device__ __forceinline__ uint32_t choisir(const uint32_t (&a)[3], uint32_t j) {
    return j == 0 ? a[0] : (j == 1 ? a[1] : a[2]);
}

__host__ __device__ inline Disposition disposition(const Dims& d, uint32_t j) {
    uint64_t base = 0;
    for (uint32_t i = 0; i < 3; ++i)
        if (i < j) base += disposition_matrice(d.lignes[i], d.colonnes[i]).pas;
    Disposition r = disposition_matrice(choisir(d.lignes, j), choisir(d.colonnes, j));
    r.base = base;
    return r;
}

// ------------------------------------------------------------------ parts and streams

struct Flux {
    const uint8_t* p;    // stream start (16-aligned when the part is)
    uint32_t longueur;   // stream bytes
    uint32_t produits;   // bytes its decoding produces (stream table)
};

// First stream (sorte, matrice) of a level-0 part of `taille` bytes (at least 64), with the
// structural checks the kernels can afford (trouver_flux, commun.cuh:111-129 of the reference,
// plus the part size the host knows): magic and level 0, stream table and stream inside the
// useful bytes, useful bytes inside the buffer, stream offset 16-aligned.
__device__ inline bool trouver_flux(const uint8_t* partie, uint64_t taille, uint8_t sorte, uint32_t matrice, Flux& f) {
    const uint4 tete = *reinterpret_cast<const uint4*>(partie);
    if (tete.x != MAGIE_PARTIE0) return false;
    if ((tete.z & 0xFFu) != 0) return false;  // level 0
    const uint32_t n_flux = tete.z >> 16;
    const uint32_t utiles = tete.w;
    if (utiles > taille || n_flux > 255u || 64u + 16u * n_flux > utiles) return false;
    for (uint32_t i = 0; i < n_flux; ++i) {
        const uint4 e = *reinterpret_cast<const uint4*>(partie + 64 + 16 * i);
        if ((e.x & 0xFFu) == sorte && ((e.x >> 8) & 0xFFu) == matrice) {
            if ((e.y & 15u) != 0 || uint64_t(e.y) + e.z > utiles) return false;
            f.p = partie + e.y;
            f.longueur = e.z;
            f.produits = e.w;
            return true;
        }
    }
    return false;
}

// The same lookup by a whole warp: lane l reads descriptors l, l + 32, ... together (one round
// trip for up to 32 streams, where trouver_flux waits for one descriptor after the other). Every
// lane of a converged warp calls it with the same arguments and gets the same result.
__device__ inline bool trouver_flux_warp(const uint8_t* partie, uint64_t taille, uint8_t sorte, uint32_t matrice,
                                         Flux& f) {
    const uint32_t voie = threadIdx.x & 31u;
    const uint4 tete = *reinterpret_cast<const uint4*>(partie);
    if (tete.x != MAGIE_PARTIE0) return false;
    if ((tete.z & 0xFFu) != 0) return false;  // level 0
    const uint32_t n_flux = tete.z >> 16;
    const uint32_t utiles = tete.w;
    if (utiles > taille || n_flux > 255u || 64u + 16u * n_flux > utiles) return false;
    for (uint32_t base = 0; base < n_flux; base += 32u) {
        const uint32_t i = base + voie;
        const uint4 e = i < n_flux ? *reinterpret_cast<const uint4*>(partie + 64 + 16 * i) : make_uint4(0u, 0u, 0u, 0u);
        const bool ok = i < n_flux && (e.x & 0xFFu) == sorte && ((e.x >> 8) & 0xFFu) == matrice;
        const uint32_t v = __ballot_sync(0xFFFFFFFFu, ok);
        if (v != 0) {
            const int src = __ffs(v) - 1;
            const uint32_t dec = __shfl_sync(0xFFFFFFFFu, e.y, src);
            const uint32_t lon = __shfl_sync(0xFFFFFFFFu, e.z, src);
            const uint32_t pro = __shfl_sync(0xFFFFFFFFu, e.w, src);
            if ((dec & 15u) != 0 || uint64_t(dec) + lon > utiles) return false;
            f.p = partie + dec;
            f.longueur = lon;
            f.produits = pro;
            return true;
        }
    }
    return false;
}

// A validated rANS stream header (rans.rs:231-280; commun.cuh:146-165 of the reference).
struct EnteteRans {
    uint32_t P, N, T, W;
    const uint32_t* debut;  // T tile starts (word indices)
    const uint32_t* etats;  // 32 T lane states
    const uint8_t* mots;    // words u16[W] (4-byte aligned)
};

// `besoin`: the useful bytes the stream must produce; P is besoin rounded up to 128.
__device__ inline bool lire_entete(const Flux& f, uint32_t besoin, EnteteRans& h) {
    if (f.longueur < 16) return false;
    const uint4 t = *reinterpret_cast<const uint4*>(f.p);
    h.P = t.x;
    h.N = t.y & 0xFFFFu;
    const uint32_t geo = (t.y >> 16) & 0xFFu, reserve = t.y >> 24;
    h.T = t.z;
    h.W = t.w;
    if (geo != 1u || reserve != 0 || h.N == 0 || (h.P & 127u) != 0) return false;
    if (h.P < besoin || h.P - besoin >= 128u) return false;
    if (f.produits != h.P && f.produits != besoin) return false;
    const uint32_t macro = h.P / 128u;
    if (h.T != (macro + h.N - 1) / h.N) return false;
    if (16ull + 132ull * h.T + 2ull * h.W > f.longueur) return false;
    h.debut = reinterpret_cast<const uint32_t*>(f.p + 16);
    h.etats = reinterpret_cast<const uint32_t*>(f.p + 16 + 4ull * h.T);
    h.mots = f.p + 16 + 132ull * h.T;
    return true;
}

// ------------------------------------------------------------------ programmatic dependent launch

// Waits until the previous kernel on the stream has completed and its writes are visible (a no-op
// when the kernel was not launched with programmatic serialization).
__device__ __forceinline__ void attendre_amont() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
// Lets the next kernel on the stream start its prologue.
__device__ __forceinline__ void liberer_aval() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

// ------------------------------------------------------------------ mbarriers (shared memory)

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t n) {
    asm volatile("mbarrier.init.shared.b64 [%0], %1;\n" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(b))), "r"(n)
                 : "memory");
}
// Arrival with release semantics (the caller's earlier shared-memory writes are visible to a
// thread whose wait on this phase succeeds).
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared.b64 st, [%0];\n\t}" ::"r"(
                     static_cast<uint32_t>(__cvta_generic_to_shared(b)))
                 : "memory");
}
__device__ __forceinline__ bool mbar_essai(uint64_t* b, uint32_t parite) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(b))), "r"(parite)
        : "memory");
    return ok != 0;
}
// Waits until the phase of parity `parite` has completed, at most ATTENTES_MAX tries (each may
// suspend the warp for a short while); false when it gave up.
constexpr uint32_t ATTENTES_MAX = 1u << 22;
__device__ __forceinline__ bool mbar_attendre(uint64_t* b, uint32_t parite) {
    for (uint32_t n = 0; n < ATTENTES_MAX; ++n)
        if (mbar_essai(b, parite)) return true;
    return false;
}

// ------------------------------------------------------------------ async copies

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, uint32_t src_octets) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_octets) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t adresse_partagee(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ the warp decoder

// One warp decoding one tile. All fields but `x` are warp-uniform.
//
// Sub-step (the dependent chain, measured ~87 ns on B200 with one warp per SM): the LUT entry
// of the state; meanwhile every lane pre-loads the ring word at (pointer + its lane index);
// y = f (x >> 12) + b; a ballot of the lanes with y < L; the lane that renormalises takes its
// word from the lane whose index is its prefix count (one shuffle), merged by a byte permute.
struct Decodeur {
    uint32_t x;            // rANS state of this lane
    uint32_t pa;           // next word, as an aligned index (stream word index + dec)
    uint32_t fin_a;        // end of the tile's words (debut[t+1], or W for the last), aligned
    uint32_t lim;          // stream words at or past `lim` read as 0: min(fin, W)
    uint32_t dec;          // words between the 16-aligned base `ga` and mots[0]
    uint32_t tranche;      // chunk (256 aligned words from ga) the pointer is in
    const uint8_t* ga;     // 16-aligned address at or below mots[0]
    uint16_t* anneau;      // this warp's ring (ANNEAU_ALLOC words, shared memory)
    uint32_t masque_inf;   // lanes below this one
    uint32_t voie;

    // Chunk c (aligned words [256c, 256c + 256)) into its ring slot; each lane copies 16 bytes,
    // zero-filled past `lim`. The chunk landing at slot 0 is also copied into the mirror.
    __device__ __forceinline__ void charger(uint32_t c) {
        const uint32_t a0 = c * TRANCHE_MOTS + 8u * voie;   // aligned index of the lane's first word
        const int64_t i0 = int64_t(a0) - int64_t(dec);      // stream word index
        int64_t utiles = int64_t(lim) - i0;                 // words this lane may read
        utiles = utiles < 0 ? 0 : (utiles > 8 ? 8 : utiles);
        const uint8_t* src = utiles > 0 ? ga + 2ull * a0 : ga;
        const uint32_t fente = a0 & (ANNEAU_MOTS - 1u);
        cp_async16(anneau + fente, src, uint32_t(2 * utiles));
        if (fente < MIROIR_MOTS) cp_async16(anneau + ANNEAU_MOTS + fente, src, uint32_t(2 * utiles));
    }

    __device__ __forceinline__ void debut(const EnteteRans& h, uint32_t t, uint32_t v, uint16_t* ring) {
        voie = v;
        anneau = ring;
        masque_inf = (1u << voie) - 1u;
        x = h.etats[t * VOIES + voie];
        const uint32_t ptr = h.debut[t];
        const uint32_t fin = (t + 1 < h.T) ? h.debut[t + 1] : h.W;
        lim = fin < h.W ? fin : h.W;
        const uintptr_t m = reinterpret_cast<uintptr_t>(h.mots);
        ga = reinterpret_cast<const uint8_t*>(m & ~uintptr_t(15));
        dec = uint32_t(m & 15u) >> 1;
        pa = ptr + dec;
        fin_a = fin + dec;
        tranche = pa / TRANCHE_MOTS;
        __syncwarp();
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) {
            charger(tranche + c);
            cp_async_commit();
        }
        cp_async_wait<2>();
        __syncwarp();
    }

    // At the start of each macro-step: when the pointer entered a new chunk, refill the slot
    // of the chunk left behind with the chunk three ahead, and make sure the current and next
    // chunks (all this macro-step can read: at most 128 words) have landed.
    __device__ __forceinline__ void avancer() {
        const uint32_t c = pa / TRANCHE_MOTS;
        if (c != tranche) {
            tranche = c;
            __syncwarp();
            charger(c + 3u);
            cp_async_commit();
            cp_async_wait<2>();
            __syncwarp();
        }
    }

    // One sub-step; `lut`: the table in shared memory. Returns the LUT entry (its low byte is
    // the symbol). Plain loads (not volatile asm): the compiler schedules them, and they stay
    // ordered after the ring refill's wait (a memory clobber).
    __device__ __forceinline__ uint32_t pas(const uint32_t* lut) {
        const uint32_t e = lut[x & (M - 1u)];
        const uint32_t pre = anneau[(pa & (ANNEAU_MOTS - 1u)) + voie];
        const uint32_t y = (((e >> 8) & 0xFFFu) + 1u) * (x >> 12) + (e >> 20);
        const bool besoin = y < L;
        const uint32_t vote = __ballot_sync(0xFFFFFFFFu, besoin);
        const uint32_t w = __shfl_sync(0xFFFFFFFFu, pre, __popc(vote & masque_inf));
        x = besoin ? __byte_perm(w, y, 0x5410) : y;
        pa += __popc(vote);
        return e;
    }

    // Four sub-steps: the lane's 32-bit output word (byte k = sub-step k).
    __device__ __forceinline__ uint32_t macro(const uint32_t* lut) {
        uint32_t m = pas(lut);
        m = __byte_perm(m, pas(lut), 0x0040);
        m = __byte_perm(m, pas(lut), 0x0410);
        m = __byte_perm(m, pas(lut), 0x4210);
        return m;
    }

    // Four sub-steps, with the caller's independent work f(Etape<k>) placed after sub-step k:
    // it fills the decode chain's latency instead of following it.
    template <typename F>
    __device__ __forceinline__ uint32_t macro(const uint32_t* lut, F&& f) {
        uint32_t m = pas(lut);
        f(Etape<0>{});
        m = __byte_perm(m, pas(lut), 0x0040);
        f(Etape<1>{});
        m = __byte_perm(m, pas(lut), 0x0410);
        f(Etape<2>{});
        m = __byte_perm(m, pas(lut), 0x4210);
        f(Etape<3>{});
        return m;
    }

    // ---- look-ahead form, for streams whose lanes all read one table (DELTA) ----
    // The sub-step above waits for the LUT entry of the new state before the next one starts.
    // Here every lane carries, besides the LUT entry `e` of its state, the ring word at
    // (pointer + lane) and that word's LUT entry: a lane that renormalises takes both from the
    // lane of its rank (two shuffles), a lane that does not has the entry of y in flight since y
    // was known, so the table lookup overlaps the ballot and shuffle instead of following them.
    // The words are those of pas(), in the same order: the same states, bytes and pointer.
    // The ring word of a macro-step's first sub-step is read at the end of the previous one,
    // before avancer(): at most 128 + 31 words past that macro-step's start, so inside the
    // chunk after the pointer's, which avancer() keeps landed; the chunk avancer() refills is
    // behind the pointer.
    struct Avance {
        uint32_t e, wp, lp;
    };

    // After debut(): the first sub-step's entries.
    __device__ __forceinline__ void debut_avance(const uint32_t* lut, Avance& s) {
        s.e = lut[x & (M - 1u)];
        s.wp = anneau[(pa & (ANNEAU_MOTS - 1u)) + voie];
        s.lp = lut[s.wp & (M - 1u)];
    }

    __device__ __forceinline__ uint32_t pas_avance(const uint32_t* lut, Avance& s) {
        const uint32_t e = s.e;
        const uint32_t y = (((e >> 8) & 0xFFFu) + 1u) * (x >> 12) + (e >> 20);
        const uint32_t ey = lut[y & (M - 1u)];
        const bool besoin = y < L;
        const uint32_t vote = __ballot_sync(0xFFFFFFFFu, besoin);
        const uint32_t rang = __popc(vote & masque_inf);
        const uint32_t w = __shfl_sync(0xFFFFFFFFu, s.wp, rang);
        const uint32_t ew = __shfl_sync(0xFFFFFFFFu, s.lp, rang);
        x = besoin ? __byte_perm(w, y, 0x5410) : y;
        s.e = besoin ? ew : ey;
        pa += __popc(vote);
        s.wp = anneau[(pa & (ANNEAU_MOTS - 1u)) + voie];
        s.lp = lut[s.wp & (M - 1u)];
        return e;
    }

    // The look-ahead form on the table restaged as 64-bit entries {f, i - c} (lut2, from
    // restager_lut2) with the symbols in a byte table: y = f (x >> 12) + (i - c) is one multiply-
    // add of the loaded entry, the fields no longer extracted on the chain; the symbol is read
    // beside it, off the chain. The same arithmetic as pas_avance, so the same states and bytes.
    struct Avance2 {
        uint2 e, lp;
        uint32_t wp;
    };

    __device__ __forceinline__ void debut_avance2(const uint2* lut2, Avance2& s) {
        s.e = lut2[x & (M - 1u)];
        s.wp = anneau[(pa & (ANNEAU_MOTS - 1u)) + voie];
        s.lp = lut2[s.wp & (M - 1u)];
    }

    __device__ __forceinline__ uint32_t pas_avance2(const uint2* lut2, const uint8_t* symboles, Avance2& s) {
        const uint32_t symbole = symboles[x & (M - 1u)];
        const uint32_t y = s.e.x * (x >> 12) + s.e.y;
        const uint2 ey = lut2[y & (M - 1u)];
        const bool besoin = y < L;
        const uint32_t vote = __ballot_sync(0xFFFFFFFFu, besoin);
        const uint32_t rang = __popc(vote & masque_inf);
        const uint32_t w = __shfl_sync(0xFFFFFFFFu, s.wp, rang);
        const uint32_t f = __shfl_sync(0xFFFFFFFFu, s.lp.x, rang);
        const uint32_t b = __shfl_sync(0xFFFFFFFFu, s.lp.y, rang);
        x = besoin ? __byte_perm(w, y, 0x5410) : y;
        s.e = besoin ? make_uint2(f, b) : ey;
        pa += __popc(vote);
        s.wp = anneau[(pa & (ANNEAU_MOTS - 1u)) + voie];
        s.lp = lut2[s.wp & (M - 1u)];
        return symbole;
    }

    __device__ __forceinline__ uint32_t macro_avance2(const uint2* lut2, const uint8_t* symboles, Avance2& s) {
        uint32_t m = pas_avance2(lut2, symboles, s);
        m = __byte_perm(m, pas_avance2(lut2, symboles, s), 0x0040);
        m = __byte_perm(m, pas_avance2(lut2, symboles, s), 0x0410);
        m = __byte_perm(m, pas_avance2(lut2, symboles, s), 0x4210);
        return m;
    }

    __device__ __forceinline__ uint32_t macro_avance(const uint32_t* lut, Avance& s) {
        uint32_t m = pas_avance(lut, s);
        m = __byte_perm(m, pas_avance(lut, s), 0x0040);
        m = __byte_perm(m, pas_avance(lut, s), 0x0410);
        m = __byte_perm(m, pas_avance(lut, s), 0x4210);
        return m;
    }

    // With the caller's independent work f(Etape<k>) after sub-step k (as macro(lut, f)).
    template <typename F>
    __device__ __forceinline__ uint32_t macro_avance(const uint32_t* lut, Avance& s, F&& f) {
        uint32_t m = pas_avance(lut, s);
        f(Etape<0>{});
        m = __byte_perm(m, pas_avance(lut, s), 0x0040);
        f(Etape<1>{});
        m = __byte_perm(m, pas_avance(lut, s), 0x0410);
        f(Etape<2>{});
        m = __byte_perm(m, pas_avance(lut, s), 0x4210);
        f(Etape<3>{});
        return m;
    }

    // End-of-tile integrity: lanes off L; the word pointer must end at the tile's end.
    __device__ __forceinline__ void bilan(uint32_t& hors_l, uint32_t& pointeur) const {
        hors_l += x != L ? 1u : 0u;
        pointeur += (voie == 0 && pa != fin_a) ? 1u : 0u;
    }

    // Drains the copies still in flight (the ring must not be written after the warp leaves).
    __device__ __forceinline__ void terminer() {
        cp_async_wait<0>();
        __syncwarp();
    }
};

// Rows of the blocks a lane's DELTA word covers: word w = 32 m + lane carries delta of blocks
// 4w .. 4w+3; the lane keeps the row and the position in the row of block 4w, advanced by 128
// blocks per macro-step without division or branch (q = 128 / B, r = 128 % B precomputed).
struct LignesDelta {
    uint32_t ligne, reste, B, q, r;
    __device__ __forceinline__ void debut(uint32_t b0, uint32_t B_) {
        B = B_;
        ligne = b0 / B;
        reste = b0 - ligne * B;
        q = 128u / B;
        r = 128u - q * B;
    }
    // Row of block 4w + k (B >= 4: the four blocks span at most two rows).
    __device__ __forceinline__ uint32_t rang(uint32_t k) const {
        const uint32_t qk = reste + k;
        return B >= 4u ? ligne + (qk >= B ? 1u : 0u) : ligne + qk / B;
    }
    __device__ __forceinline__ void avancer() {
        reste += r;
        ligne += q;
        const bool c = reste >= B;
        reste -= c ? B : 0u;
        ligne += c ? 1u : 0u;
    }
};

__device__ __forceinline__ uint32_t somme_warp(uint32_t v) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, d);
    return v;
}

__device__ __forceinline__ void verser_controle(uint32_t* controle, uint32_t voie, uint32_t hors_l, uint32_t pointeur) {
    hors_l = somme_warp(hors_l);
    pointeur = somme_warp(pointeur);
    if (voie == 0) {
        if (hors_l) atomicAdd(&controle[CTL_HORS_L], hors_l);
        if (pointeur) atomicAdd(&controle[CTL_POINTEUR], pointeur);
    }
}

// Matrix j of a raw part (ECHELLES_BRUTES, CODES_BRUTS, BIAIS) into its place in an SoA slot
// (grid-stride over the block's threads and gridDim.x); a missing or short stream counts a
// format error in controle[CTL_FORMAT] (block x 0).
__device__ inline void copier_brut_matrice(const uint8_t* partie, uint64_t taille, uint8_t* emplacement, const Dims& dims,
                                           uint32_t j, uint32_t* controle) {
    const uint32_t R = choisir(dims.lignes, j), C = choisir(dims.colonnes, j);
    const uint32_t B = C / 32u, nblocs = R * B;
    Flux fe, fc, fb;
    const bool bon = B > 0 && R > 0 && trouver_flux_warp(partie, taille, SORTE_ECHELLES_BRUTES, j, fe) &&
                     trouver_flux_warp(partie, taille, SORTE_CODES_BRUTS, j, fc) && trouver_flux_warp(partie, taille, SORTE_BIAIS, j, fb) &&
                     fe.produits == nblocs && fe.longueur >= nblocs && fc.produits == 16u * nblocs &&
                     fc.longueur >= 16u * nblocs && fb.produits == 4u * R && fb.longueur >= 4u * R;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const Disposition disp = disposition(dims, j);
    uint8_t* mat = emplacement + disp.base;
    const uint32_t i0 = blockIdx.x * blockDim.x + threadIdx.x, pas = gridDim.x * blockDim.x;
    const uint4* cs = reinterpret_cast<const uint4*>(fc.p);
    uint4* cd = reinterpret_cast<uint4*>(mat);
    for (uint32_t i = i0; i < nblocs; i += pas) cd[i] = cs[i];
    const uint32_t n4 = nblocs / 4u;
    const uint32_t* es = reinterpret_cast<const uint32_t*>(fe.p);
    uint32_t* ed = reinterpret_cast<uint32_t*>(mat + disp.echelles);
    for (uint32_t i = i0; i < n4; i += pas) ed[i] = es[i];
    for (uint32_t i = 4u * n4 + i0; i < nblocs; i += pas) mat[disp.echelles + i] = fe.p[i];
    const uint32_t* bs = reinterpret_cast<const uint32_t*>(fb.p);
    uint32_t* bd = reinterpret_cast<uint32_t*>(mat + disp.biais);
    for (uint32_t i = i0; i < R; i += pas) bd[i] = bs[i];
}

// Scale class of a block from its scale and its row's median (4.9.3): delta = e - med + 128.
__device__ __forceinline__ uint32_t classe_echelle(uint32_t e, uint32_t med) {
    const uint32_t d = (e - med + 128u) & 255u;
    return d < 128u ? 0u : (d == 128u ? 1u : 2u);
}

}  // namespace tb
