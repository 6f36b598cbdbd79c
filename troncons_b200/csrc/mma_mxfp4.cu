// troncons_b200 — the MXFP4 expert GEMM on the 5th-generation tensor cores, for experts that
// receive many tokens at once (a prefill batch par flux, an expert-parallel share at batch 64):
// Y[n][r] = sum_c W[r][c] X[n][c] + b[r], W an expert matrix in the slot / raw-part layout (16
// code bytes and one E8M0 scale per 32-block, row-major), X f32 or bf16 activations.
//
// tcgen05.mma.kind::mxf8f6f4.block_scale, M = 128 rows, N = the tokens (8 to 256), K = 32 per
// instruction: A = the weights as E2M1 with their own E8M0 block scales, B = the activations as
// MXFP8 (E4M3 elements, one E8M0 scale per 32, the OCP MX rule: scale = 2^(floor(log2 max|x|)
// - 8)), f32 accumulation in tensor memory. The block scales are the hardware's (one per row or
// token and 32-block, read from tensor memory); the weights are not dequantized on CUDA cores.
//
// Layout of a 32-block in the K order the MMA sees. The file stores element i of a block in the
// low nibble of byte i and element 16 + i in the high nibble. Read as a packed E2M1 vector (two
// elements per byte, the low nibble first), those 16 bytes are the block's elements in the order
// k' = 2i -> element i, k' = 2i + 1 -> element 16 + i. The MMA sums over K, so the activations are
// quantized into that same order and no weight byte is moved: the two 8-byte halves of a block
// land as they are in the unpacked shared-memory form of 4-bit operands (16 elements in 8 bytes,
// then 8 bytes of padding, per 16 bytes).
//
// Shared memory, K-major with the 128-byte swizzle: one chunk of 128 K is a [rows][128 bytes]
// tile (A: 128 weight rows, B: the tokens), the 16-byte pieces of row r at piece index XOR
// (r mod 8), 8-row atoms of 1,024 bytes; each MMA of the chunk starts 32 bytes further along K.
// The tiles come by TMA (cp.async.bulk.tensor, no multicast): A with the 4-bit unpacking tensor
// type (packed in global memory, 8 bytes of padding per 16 elements written in shared memory),
// a 3-D view (128 elements, the row's full chunks, rows) when the matrix allows it (codes
// 32-aligned, columns a multiple of 64); otherwise, and for a last partial chunk, the halves by
// 8-byte cp.async into the same swizzled places. B, the quantized activations, by a 2-D TMA
// (out-of-range tokens and columns read as zeros). Scale factors in tensor memory, the layout of
// tcgen05.cp's 32x128b copies replicated to the four lane quadrants: lane (m mod 32), column
// m / 32 + base, byte = the 32-block within the chunk (the instruction descriptor's and the
// address's scale-factor id); their words are arranged once per CTA in shared memory.
//
// One CTA of 5 warps per 128-row tile, the roles decoupled by two mbarriers per stage. Warps
// 0-3 produce: for chunk ch they wait until stage ch mod E is free (its previous chunk's MMAs
// committed); thread 0 announces the stage's TMA bytes and issues the copies; each warp writes
// its lane quadrant's scale factors to tensor memory; every producer thread then arrives on the
// stage's "full" barrier (through cp.async.mbarrier.arrive when it issued 8-byte copies, which
// lands with them). Warp 4's lane 0 issues the MMAs: it waits for "full", issues the chunk's four
// MMAs and commits them to the stage's "empty" barrier, so the copies run up to E chunks ahead of
// the MMAs. After the last chunk the MMA thread commits to a "done" barrier, on which warps 0-3
// wait to read the accumulator (tcgen05.ld), add the bias and store Y. Every wait is bounded: a
// wait that gives up sets the caller's error word and ends its role; the MMA thread always
// commits "done" (so the others know the MMAs in flight have finished), the producers drain
// their copies, and the tensor memory is freed before the CTA returns.
#include <cuda.h>  // CUtensorMap and the encoder's types (the encoder itself is resolved at run time)

#include <cstdint>
#include <cstring>

#include "commun.cuh"
#include "noyaux.h"

namespace tb {

constexpr uint32_t MMA_M = 128;        // rows per CTA (one MMA's M); chunks of 128 K (four MMAs)
constexpr uint32_t MMA_PROD = 128;     // warps 0-3: one per tensor-memory lane quadrant
constexpr uint32_t MMA_FILS = 160;     // + warp 4, the MMA issuer
constexpr uint32_t LOT_MAX = 48;       // matrices per launch (their descriptors and tensor maps are kernel parameters)

// Stages of 128 K: as many as fit (3 to 6) with two CTAs per SM, else with one.
constexpr uint32_t MMA_ETAGES_MAX = 6;

__host__ __device__ __forceinline__ uint32_t mma_n_pad(uint32_t N) { return (N + 15u) & ~15u; }
__host__ __device__ __forceinline__ uint32_t mma_chunks(uint32_t C) { return (C / 32u + 3u) / 4u; }
// Tensor-memory columns: the accumulator (Npad), then per stage SFA (4) and SFB (8).
__host__ __device__ __forceinline__ uint32_t mma_tmem_colonnes(uint32_t N, uint32_t E) {
    const uint32_t besoin = mma_n_pad(N) + 12u * E;
    uint32_t c = 32u;
    while (c < besoin) c <<= 1;
    return c;
}
// Shared bytes of one stage: A tile (128 rows x 128 bytes) and B tile (Npad rows x 128 bytes).
__host__ __device__ __forceinline__ uint32_t mma_etage(uint32_t N) { return MMA_M * 128u + mma_n_pad(N) * 128u; }
// The scale-factor words of every chunk: [chunk][128 rows, then Npad tokens].
__host__ __device__ __forceinline__ uint32_t mma_mots_ligne(uint32_t N) { return MMA_M + mma_n_pad(N) + 1u; }
__host__ __device__ __forceinline__ uint32_t mma_mots_ef(uint32_t N, uint32_t C) {
    return (mma_chunks(C) * mma_mots_ligne(N) * 4u + 15u) & ~15u;
}
// 1,024 bytes of alignment slack, the stages, the scale-factor words, the mbarriers (full and
// empty per stage, done), the tensor-memory base and the abandon flag.
__host__ __device__ __forceinline__ uint32_t mma_smem(uint32_t N, uint32_t C, uint32_t E) {
    return 1024u + E * mma_etage(N) + mma_mots_ef(N, C) + 16u * E + 16u;
}
// The stage count that keeps the most chunks in flight per SM (CTAs per SM x stages, up to
// three CTAs; on a tie, more CTAs: their prologues and epilogues overlap each other's copies).
__host__ __device__ inline uint32_t mma_etages(uint32_t N, uint32_t C) {
    uint32_t meilleur = 3u, total = 0u;
    for (uint32_t E = 3u; E <= MMA_ETAGES_MAX && mma_smem(N, C, E) <= 220u * 1024u; ++E) {
        const uint32_t ctas = min(3u, (228u * 1024u) / (mma_smem(N, C, E) + 1024u));
        if (ctas * E > total) {
            total = ctas * E;
            meilleur = E;
        }
    }
    return meilleur;
}

// Offset of byte k (0..127) of row r in a [rows][128] tile with the 128-byte swizzle.
__device__ __forceinline__ uint32_t mma_off(uint32_t r, uint32_t k) {
    return r * 128u + ((((k >> 4) ^ (r & 7u)) << 4) | (k & 15u));
}

// Shared-memory matrix descriptor, K-major with the 128-byte swizzle: stride between 8-row
// groups 1,024 bytes; the leading offset is unused in this mode (1).
__device__ __forceinline__ uint64_t mma_desc(uint32_t adresse) {
    uint64_t d = 0;
    d |= uint64_t((adresse >> 4) & 0x3FFFu);
    d |= uint64_t(1) << 16;           // leading byte offset (unused)
    d |= uint64_t(1024u >> 4) << 32;  // stride byte offset: the next 8 rows
    d |= uint64_t(1) << 46;           // descriptor version of sm_100
    d |= uint64_t(2) << 61;           // 128-byte swizzle
    return d;                         // base offset 0: tiles are 1,024-aligned
}

// Instruction descriptor: E2M1 A, E4M3 B, f32 D, K-major both, E8M0 scales, M = 128, N.
__device__ __forceinline__ uint32_t mma_idesc(uint32_t N, uint32_t sf) {
    uint32_t d = 0;
    d |= (sf & 3u) << 4;          // B scale-factor id
    d |= 5u << 7;                 // A: E2M1
    d |= 0u << 10;                // B: E4M3
    d |= (N >> 3) << 17;          // N / 8
    d |= 1u << 23;                // scale format E8M0
    d |= (MMA_M >> 4) << 24;      // M / 16
    d |= (sf & 3u) << 29;         // A scale-factor id
    return d;
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(adresse_partagee(smem)), "l"(gmem) : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(taddr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr)
                 : "memory");
}

// The thread's cp.async copies issued so far arrive on mbarrier b when they have landed (one
// arrival of the barrier's expected count, not an added one).
__device__ __forceinline__ void cp_async_arriver(uint64_t* b) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(adresse_partagee(b)) : "memory");
}
__device__ __forceinline__ void mbar_octets_attendus(uint64_t* b, uint32_t octets) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;\n" ::"r"(adresse_partagee(b)), "r"(octets)
                 : "memory");
}
// TMA loads onto mbarrier b (this CTA's shared memory; no multicast).
__device__ __forceinline__ void tma_3d(void* dst, const CUtensorMap* carte, int32_t c0, int32_t c1, int32_t c2, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(
            adresse_partagee(dst)),
        "l"(reinterpret_cast<uint64_t>(carte)), "r"(c0), "r"(c1), "r"(c2), "r"(adresse_partagee(b))
        : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* carte, int32_t c0, int32_t c1, uint64_t* b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
            adresse_partagee(dst)),
        "l"(reinterpret_cast<uint64_t>(carte)), "r"(c0), "r"(c1), "r"(adresse_partagee(b))
        : "memory");
}

// The weight halves of rows r0 .. r0 + 127, 32-blocks kb0 .. kb0 + nkb - 1, into the A tile by
// 8-byte copies (producer threads).
__device__ __forceinline__ void charger_a(uint8_t* ta, const uint8_t* codes, uint32_t R, uint32_t B, uint32_t r0,
                                          uint32_t kb0, uint32_t nkb) {
    for (uint32_t t = threadIdx.x; t < MMA_M * 4u * 2u; t += MMA_PROD) {
        const uint32_t r = t >> 3, kb = (t >> 1) & 3u, h = t & 1u;
        if (kb >= nkb || r0 + r >= R) continue;
        const uint8_t* src = codes + (uint64_t(r0 + r) * B + kb0 + kb) * 16u + 8u * h;
        cp_async8(ta + mma_off(r, 32u * kb + 16u * h), src);
    }
}

// The quantized activations of the chunk (32 bytes per token and block) into the B tile by
// 16-byte copies (when the matrix's B tile cannot come by TMA).
__device__ __forceinline__ void charger_b(uint8_t* tb_, const uint8_t* xq, uint32_t C, uint32_t N, uint32_t kb0,
                                          uint32_t nkb) {
    for (uint32_t t = threadIdx.x; t < N * 4u * 2u; t += MMA_PROD) {
        const uint32_t n = t >> 3, kb = (t >> 1) & 3u, h = t & 1u;
        if (kb >= nkb) continue;
        cp_async16(tb_ + mma_off(n, 32u * kb + 16u * h), xq + uint64_t(n) * C + 32u * (kb0 + kb) + 16u * h, 16u);
    }
}

// A batch of GEMMs in one launch (grid y = the matrix): descriptors and tensor maps as kernel
// parameters, the quantized x of matrix i at espace + (premier + i) tranche.
struct LotMma {
    CUtensorMap ta[LOT_MAX];   // A: 4-bit unpacking, (128, full chunks, rows)
    CUtensorMap tb[LOT_MAX];   // B: bytes, (columns, tokens)
    DescGemm d[LOT_MAX];
    RenvoiGemm r[LOT_MAX];     // token n's x row and y row (gathered / scattered), or n and n
    uint8_t* espace;
    uint32_t* erreur;
    uint64_t tranche;
    uint64_t tma_a, tma_b;     // bit i: matrix i's A (B) tiles by TMA
    uint32_t nb, premier;
};

__global__ void __launch_bounds__(MMA_FILS, 3) k_gemm_mxfp4(const __grid_constant__ LotMma lot, uint32_t E) {
    extern __shared__ __align__(1024) uint8_t dyn_brut[];
    uint8_t* dyn = dyn_brut + ((1024u - (adresse_partagee(dyn_brut) & 1023u)) & 1023u);  // 1,024-aligned tiles
    const uint32_t m = blockIdx.y;
    const DescGemm& d = lot.d[m];
    const uint32_t R = d.lignes, C = d.colonnes, N = d.n;
    if (blockIdx.x * MMA_M >= R || N == 0) return;
    const uint8_t* codes = reinterpret_cast<const uint8_t*>(d.codes);
    const uint8_t* ech = reinterpret_cast<const uint8_t*>(d.echelles);
    const float* biais = reinterpret_cast<const float*>(d.biais);
    float* y = reinterpret_cast<float*>(d.y);
    const uint8_t* xq = lot.espace + (uint64_t(lot.premier) + m) * lot.tranche;
    const uint8_t* xs = xq + uint64_t(mma_n_pad(N)) * C;
    const bool tma_a = (lot.tma_a >> m) & 1u, tma_b = (lot.tma_b >> m) & 1u;
    const uint32_t Np = mma_n_pad(N), etage = mma_etage(N), B = C / 32u;
    const uint32_t nchunks = mma_chunks(C), pleins = C / 128u;  // chunks of 128 K; those with no partial block
    uint32_t* mots = reinterpret_cast<uint32_t*>(dyn + E * etage);  // scale-factor words [chunk][128 + Np]
    uint64_t* plein = reinterpret_cast<uint64_t*>(dyn + E * etage + mma_mots_ef(N, C));
    uint64_t* vide = plein + E;
    uint64_t* fini = vide + E;
    uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(fini + 1);
    volatile uint32_t* abandon = tmem_base_s + 1;  // a role gave up: the others stop
    const uint32_t warp = threadIdx.x >> 5, voie = threadIdx.x & 31u;
    const uint32_t r0 = blockIdx.x * MMA_M;
    const uint32_t ncol = mma_tmem_colonnes(N, E);
    const uint32_t col_acc = 0;
    auto col_sfa = [Np](uint32_t e) { return Np + 12u * e; };
    auto col_sfb = [Np](uint32_t e) { return Np + 12u * e + 4u; };

    if (threadIdx.x == 0) {
        if (tma_a) asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&lot.ta[m])) : "memory");
        if (tma_b) asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&lot.tb[m])) : "memory");
    }
    // Stage tiles zeroed (the 8-byte copies write only data halves and rows that exist), then
    // ordered before the TMA writes that follow.
    for (uint32_t i = threadIdx.x; i < E * etage / 16u; i += MMA_FILS)
        reinterpret_cast<uint4*>(dyn)[i] = make_uint4(0, 0, 0, 0);
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
    if (threadIdx.x == 0) {
        for (uint32_t e = 0; e < E; ++e) {
            mbar_init(plein + e, MMA_PROD);  // one arrival per producer thread
            mbar_init(vide + e, 1u);         // the stage's MMAs committed
        }
        mbar_init(fini, 1u);
        *abandon = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                         adresse_partagee(tmem_base_s)),
                     "r"(ncol)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    const uint32_t tmem = *tmem_base_s;
    // Parity of the k-th completion (k = ch / E) of stage ch % E's barriers.
    auto parite = [E](uint32_t ch) { return (ch / E) & 1u; };
    const uint32_t L = mma_mots_ligne(N);  // words per chunk (odd: the scattered stores spread over the banks)
    // Stage ch's TMA copies (thread 0): the bytes announced on its "full" barrier, then issued.
    auto tma = [&](uint32_t ch) {
        const uint32_t e = ch % E;
        const bool a_tma = tma_a && ch < pleins;
        if (!a_tma && !tma_b) return;
        uint8_t* ta = dyn + e * etage;
        // The 4-bit unpacking copy counts the bytes it reads (64 per row of 128 elements), not
        // the 128 per row it writes with the padding.
        mbar_octets_attendus(plein + e, (a_tma ? MMA_M * 64u : 0u) + (tma_b ? Np * 128u : 0u));
        if (a_tma) tma_3d(ta, &lot.ta[m], 0, int32_t(ch), int32_t(r0), plein + e);
        if (tma_b) tma_2d(ta + MMA_M * 128u, &lot.tb[m], int32_t(128u * ch), 0, plein + e);
    };
    // Scale-factor words of every chunk: word (ch, m) = the E8M0 bytes of blocks 4 ch .. 4 ch + 3
    // of row m (0 past the row's blocks or past R); the tokens' words come as the quantizer
    // wrote them ([chunk][Npad], zero past their blocks). The weights' bytes are a layer input:
    // their loads are issued before the wait for the quantizer, and the first stages' copies
    // are issued while they are in flight (ahead of the copies, they do not queue behind them).
    {
        const uint32_t lignes = min(MMA_M, R - r0);
        // The CTA's rows' scale bytes are contiguous (rows r0 .. r0 + lignes - 1): consecutive
        // threads take consecutive (row, chunk) words, each read as the aligned 32-bit words it
        // straddles (coalesced; the scales are 16-aligned) and shifted into place; no read past
        // the matrix's last scale byte.
        {
            const uint64_t base = uint64_t(r0) * B, fin = uint64_t(R) * B;
            const uint32_t* e32 = reinterpret_cast<const uint32_t*>(ech);
            constexpr uint32_t LOT = 24;  // all of a 2,880-column tile's words in one round trip
            for (uint32_t t0 = threadIdx.x; t0 < lignes * nchunks; t0 += LOT * MMA_FILS) {
                uint32_t lo[LOT], hi[LOT];
#pragma unroll
                for (uint32_t k = 0; k < LOT; ++k) {
                    const uint32_t t = t0 + k * MMA_FILS;
                    const uint32_t mm = t / nchunks, ch = t - mm * nchunks;
                    const uint64_t o = base + uint64_t(mm) * B + 4u * ch;
                    lo[k] = t < lignes * nchunks ? __ldg(e32 + (o >> 2)) : 0u;
                    hi[k] = (t < lignes * nchunks && (o & 3u) != 0 && ((o >> 2) + 1u) * 4u < fin) ? __ldg(e32 + (o >> 2) + 1u) : 0u;
                }
                if (t0 == threadIdx.x) {  // first round: the activations, then the first copies
                    attendre_amont();      // the quantized activations and their scales
                    liberer_aval();
                    if (threadIdx.x == 0)
                        for (uint32_t ch = 0; ch < min(E, nchunks); ++ch) tma(ch);
                }
#pragma unroll
                for (uint32_t k = 0; k < LOT; ++k) {
                    const uint32_t t = t0 + k * MMA_FILS;
                    if (t >= lignes * nchunks) break;
                    const uint32_t mm = t / nchunks, ch = t - mm * nchunks;
                    const uint64_t o = base + uint64_t(mm) * B + 4u * ch;
                    uint32_t v = __funnelshift_r(lo[k], hi[k], 8u * uint32_t(o & 3u));
                    if (4u * ch + 4u > B) v &= (1u << (8u * (B - 4u * ch))) - 1u;  // bytes past the row's blocks
                    mots[ch * L + mm] = v;
                }
            }
            if (threadIdx.x >= lignes * nchunks) {  // a thread with no row word still waits, and thread 0 still copies
                attendre_amont();
                liberer_aval();
                if (threadIdx.x == 0)
                    for (uint32_t ch = 0; ch < min(E, nchunks); ++ch) tma(ch);
            }
            for (uint32_t t = lignes * nchunks + threadIdx.x; t < MMA_M * nchunks; t += MMA_FILS) {
                const uint32_t mm = t / nchunks, ch = t - mm * nchunks;
                mots[ch * L + mm] = 0u;  // rows past R
            }
        }
        const uint32_t* xsw = reinterpret_cast<const uint32_t*>(xs);
        constexpr uint32_t LOTW = 4;
        for (uint32_t w0 = threadIdx.x; w0 < nchunks * Np; w0 += LOTW * MMA_FILS) {
            uint32_t v[LOTW];
#pragma unroll
            for (uint32_t k = 0; k < LOTW; ++k) {
                const uint32_t w = w0 + k * MMA_FILS;
                v[k] = (w < nchunks * Np && w % Np < N) ? __ldg(xsw + w) : 0u;
            }
#pragma unroll
            for (uint32_t k = 0; k < LOTW; ++k) {
                const uint32_t w = w0 + k * MMA_FILS;
                if (w < nchunks * Np) mots[(w / Np) * L + MMA_M + w % Np] = v[k];
            }
        }
    }
    __syncthreads();

    if (warp < 4u) {
        // ---------------- producers: copies and scale factors, up to E chunks ahead
        const uint32_t quadrant = warp * 32u;
        for (uint32_t ch = 0; ch < nchunks; ++ch) {
            const uint32_t e = ch % E, kb0 = 4u * ch, nkb = min(4u, B - kb0);
            // The stage's previous chunk (ch - E): its MMAs read the tiles and the scale factors.
            // The decision is the warp's (the tcgen05 stores below are warp-wide).
            const bool libre = __all_sync(0xFFFFFFFFu, ch < E || mbar_attendre(vide + e, parite(ch - E)));
            if (!libre) *abandon = 1u;
            if (__any_sync(0xFFFFFFFFu, *abandon != 0u)) break;
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            uint8_t* ta = dyn + e * etage;
            uint8_t* tbt = ta + MMA_M * 128u;
            const bool a_tma = tma_a && ch < pleins;
            if (threadIdx.x == 0 && ch >= E) tma(ch);
            if (!a_tma) charger_a(ta, codes, R, B, r0, kb0, nkb);
            if (!tma_b) charger_b(tbt, xq, C, N, kb0, nkb);
            const uint32_t* mc = mots + ch * L;
            __syncwarp();  // the tcgen05 stores are warp-wide
            tmem_st4(tmem + (quadrant << 16) + col_sfa(e), mc[voie], mc[voie + 32u], mc[voie + 64u], mc[voie + 96u]);
            tmem_st4(tmem + (quadrant << 16) + col_sfb(e), mc[MMA_M + voie], Np > 32u ? mc[MMA_M + voie + 32u] : 0u,
                     Np > 64u ? mc[MMA_M + voie + 64u] : 0u, Np > 96u ? mc[MMA_M + voie + 96u] : 0u);
            if (Np > 128u)  // tokens 128 .. 255: four more columns
                tmem_st4(tmem + (quadrant << 16) + col_sfb(e) + 4u, mc[MMA_M + 128u + voie],
                         Np > 160u ? mc[MMA_M + 160u + voie] : 0u, Np > 192u ? mc[MMA_M + 192u + voie] : 0u,
                         Np > 224u ? mc[MMA_M + 224u + voie] : 0u);
            asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
            if (!a_tma || !tma_b)
                cp_async_arriver(plein + e);  // lands with this thread's copies of the chunk
            else
                mbar_arrive(plein + e);
        }
        cp_async_wait<0>();
    } else if (voie == 0) {
        // ---------------- the MMA issuer
        for (uint32_t ch = 0; ch < nchunks; ++ch) {
            const uint32_t e = ch % E, nkb = min(4u, B - 4u * ch);
            if (!mbar_attendre(plein + e, parite(ch))) {
                *abandon = 1u;
                break;
            }
            if (*abandon != 0u) break;
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // 8-byte copies, seen by the tensor core
            const uint32_t ta = adresse_partagee(dyn + e * etage), tbs = ta + MMA_M * 128u;
            for (uint32_t kb = 0; kb < nkb; ++kb) {
                const uint64_t da = mma_desc(ta + 32u * kb);
                const uint64_t db = mma_desc(tbs + 32u * kb);
                const uint32_t idesc = mma_idesc(Np, kb);
                const uint32_t sfa = tmem + col_sfa(e) + (kb << 30), sfb = tmem + col_sfb(e) + (kb << 30);
                const uint32_t acc = (ch > 0 || kb > 0) ? 1u : 0u;
                asm volatile(
                    "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                    "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}\n" ::"r"(
                        tmem + col_acc),
                    "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
                    : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                             adresse_partagee(vide + e))
                         : "memory");
        }
        // Every MMA issued, completed or not: "done" lands when they have (also after an abandon).
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                         adresse_partagee(fini))
                     : "memory");
    }
    __syncwarp();
    // The accumulator (or, after an abandon, the MMAs in flight) once the MMAs have completed;
    // the decision is the warp's (tcgen05.ld is warp-wide).
    const bool ok = __all_sync(0xFFFFFFFFu, mbar_attendre(fini, 0u) && *abandon == 0u);
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    if (!ok) {
        if (voie == 0) atomicExch(lot.erreur, 1u);
    } else if (warp < 4u) {
        // Epilogue: warp q reads rows r0 + 32 q + lane, 8 tokens at a time.
        const uint32_t quadrant = warp * 32u;
        const uint32_t r = r0 + quadrant + voie;
        const float bias = (biais != nullptr && r < R) ? biais[r] : 0.0f;
        for (uint32_t n0 = 0; n0 < Np; n0 += 8u) {
            uint32_t v[8];
            tmem_ld8(tmem + (quadrant << 16) + col_acc + n0, v);
            asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
            if (r < R)
                for (uint32_t j = 0; j < 8u; ++j)
                    if (n0 + j < N) {
                        const uint32_t ligne = lot.r[m].iy != nullptr ? lot.r[m].iy[n0 + j] : n0 + j;  // the token's y row
                        y[uint64_t(ligne) * R + r] = __uint_as_float(v[j]) + bias;
                    }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(ncol) : "memory");
    }
}

// X (f32 or bf16, [N][C]) of matrix blockIdx.y into MXFP8: per token and 32-block, E =
// floor(log2 max|x|) - 8 (the largest E4M3 exponent), scale byte E + 127 (E = -127 for an
// all-zero block), elements x / 2^E rounded to E4M3 (nearest even, saturating at 448), written
// in the block's MMA order (k' = 2i <- element i, k' = 2i + 1 <- element 16 + i). One warp per
// (token, block).
__global__ void __launch_bounds__(256) k_quantifier_mxfp8(const __grid_constant__ LotMma lot) {
    attendre_amont();
    liberer_aval();
    const DescGemm& d = lot.d[blockIdx.y];
    const uint32_t C = d.colonnes, N = d.n, bf16 = d.x_bf16;
    const void* x = reinterpret_cast<const void*>(d.x);
    uint8_t* xq = lot.espace + (uint64_t(lot.premier) + blockIdx.y) * lot.tranche;
    uint8_t* xs = xq + uint64_t(mma_n_pad(N)) * C;
    const uint32_t B = C / 32u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5), voie = threadIdx.x & 31u;
    if (w >= N * B) return;
    const uint32_t n = w / B, b = w % B;
    const RenvoiGemm& rv = lot.r[blockIdx.y];
    const uint32_t ligne = rv.ix != nullptr ? rv.ix[n] / rv.div_x : n;  // the token's x row
    const uint64_t i = uint64_t(ligne) * C + 32u * b + voie;
    const float v = bf16 ? __uint_as_float(uint32_t(static_cast<const uint16_t*>(x)[i]) << 16) : static_cast<const float*>(x)[i];
    float mx = fabsf(v);
#pragma unroll
    for (int k = 16; k > 0; k >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, k));
    int E = -127;
    if (mx > 0.0f) {
        const int em = int((__float_as_uint(mx) >> 23) & 255u) - 127;  // floor(log2 mx) (subnormals: -127)
        E = max(-127, min(127, em - 8));
    }
    const float q = v * __uint_as_float(uint32_t(127 - E) << 23);  // x / 2^E, exact (|E| <= 127)
    uint16_t paire;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(paire) : "f"(0.0f), "f"(q));
    const uint32_t kp = voie < 16u ? 2u * voie : 2u * (voie - 16u) + 1u;
    xq[uint64_t(n) * C + 32u * b + kp] = uint8_t(paire & 0xFFu);
    // the token's scale bytes as scale-factor words: [chunk][Npad] u32, byte = the block in its
    // chunk; the last word's bytes past the row's blocks are zero
    if (voie == 0) xs[(uint64_t(b / 4u) * mma_n_pad(N) + n) * 4u + (b & 3u)] = uint8_t(E + 127);
    if (voie == 1 && b == B - 1u)
        for (uint32_t k = (b & 3u) + 1u; k < 4u; ++k) xs[(uint64_t(b / 4u) * mma_n_pad(N) + n) * 4u + k] = 0;
}

bool gemm_mxfp4_possible(uint32_t C, uint32_t N) { return mma_smem(N, C, 3u) <= 220u * 1024u; }

// The quantized activations [Npad][C] and their scale-factor words [chunk][Npad].
uint64_t gemm_mxfp4_espace(uint32_t C, uint32_t N) {
    return uint64_t(mma_n_pad(N)) * C + uint64_t(mma_chunks(C)) * mma_n_pad(N) * 4u;
}

// ------------------------------------------------------------------ tensor maps (host)

namespace {

using EncoderTuile = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, found through the runtime (no link against the driver library).
EncoderTuile encodeur() {
    static EncoderTuile f = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncoderTuile>(nullptr);
        return reinterpret_cast<EncoderTuile>(p);
    }();
    return f;
}

// A's map: the packed codes as (128 elements, the row's full chunks, rows), 4-bit elements
// unpacked to 16 bytes per 16 in shared memory, the 128-byte swizzle. False when the matrix does
// not meet the type's rules (codes 32-aligned, row bytes a multiple of 32, one full chunk at least).
bool carte_a(CUtensorMap* t, const DescGemm& d) {
    const EncoderTuile enc = encodeur();
    const uint32_t pleins = d.colonnes / 128u;
    if (enc == nullptr || d.codes % 32u != 0 || (d.colonnes / 2u) % 32u != 0 || pleins == 0) return false;
    const cuuint64_t dims[3] = {128u, pleins, d.lignes};
    const cuuint64_t pas[2] = {64u, d.colonnes / 2u};  // bytes: the next chunk, the next row
    const cuuint32_t boite[3] = {128u, 1u, MMA_M};
    const cuuint32_t un[3] = {1u, 1u, 1u};
    return enc(t, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, 3, reinterpret_cast<void*>(d.codes), dims, pas, boite, un,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// B's map: the quantized activations as (columns, tokens) bytes, boxes of (128, Npad), the
// 128-byte swizzle; tokens past N and columns past C read as zeros.
bool carte_b(CUtensorMap* t, const uint8_t* xq, uint32_t C, uint32_t N) {
    const EncoderTuile enc = encodeur();
    if (enc == nullptr || reinterpret_cast<uintptr_t>(xq) % 16u != 0 || C % 16u != 0) return false;
    const cuuint64_t dims[2] = {C, N};
    const cuuint64_t pas[1] = {C};
    const cuuint32_t boite[2] = {128u, mma_n_pad(N)};
    const cuuint32_t un[2] = {1u, 1u};
    return enc(t, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(xq), dims, pas, boite, un,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// A batch of nb matrices (host descriptors; rows, columns and tokens of each at most lignes_max,
// colonnes_max, n_max): per group of up to LOT_MAX matrices, one launch quantizes every x into
// its workspace slice, one launch runs every matrix's row tiles (grid y = the matrix).
cudaError_t lancer_gemm_mxfp4_lot(const DescGemm* descs, uint32_t nb, uint32_t lignes_max, uint32_t colonnes_max,
                                  uint32_t n_max, uint8_t* espace, uint32_t* erreur, cudaStream_t flux,
                                  const RenvoiGemm* renvois) {
    const uint64_t tranche = (gemm_mxfp4_espace(colonnes_max, n_max) + 255u) & ~uint64_t(255);
    const uint32_t E = mma_etages(n_max, colonnes_max), smem = mma_smem(n_max, colonnes_max, E);
    cudaError_t e = assurer_smem(reinterpret_cast<const void*>(k_gemm_mxfp4), int(smem));
    if (e != cudaSuccess) return e;
    static_assert(sizeof(LotMma) <= 32000, "kernel parameters");
    LotMma* lot = new LotMma;
    for (uint32_t p = 0; p < nb && e == cudaSuccess; p += LOT_MAX) {
        memset(static_cast<void*>(lot), 0, sizeof(LotMma));
        lot->nb = std::min(LOT_MAX, nb - p);
        lot->premier = p;
        lot->espace = espace;
        lot->erreur = erreur;
        lot->tranche = tranche;
        for (uint32_t i = 0; i < lot->nb; ++i) {
            const DescGemm& d = descs[p + i];
            lot->d[i] = d;
            lot->r[i] = renvois != nullptr ? renvois[p + i] : RenvoiGemm{nullptr, nullptr, 1u};
            const uint8_t* xq = espace + uint64_t(p + i) * tranche;
            if (carte_a(&lot->ta[i], d)) lot->tma_a |= uint64_t(1) << i;
            if (carte_b(&lot->tb[i], xq, d.colonnes, d.n)) lot->tma_b |= uint64_t(1) << i;
        }
        const uint32_t B = colonnes_max / 32u;
        e = lancer_pdl(k_quantifier_mxfp8, dim3((n_max * B + 7u) / 8u, lot->nb), dim3(256), 0, flux, *lot);
        if (e == cudaSuccess)
            e = lancer_pdl(k_gemm_mxfp4, dim3((lignes_max + MMA_M - 1) / MMA_M, lot->nb), dim3(MMA_FILS), smem, flux, *lot, E);
    }
    delete lot;
    return e;
}

cudaError_t lancer_gemm_mxfp4(const uint8_t* codes, const uint8_t* ech, const float* biais, const void* x, uint32_t x_bf16,
                              float* y, uint32_t R, uint32_t C, uint32_t N, uint8_t* espace, uint32_t* erreur,
                              cudaStream_t flux) {
    DescGemm d{reinterpret_cast<uint64_t>(codes), reinterpret_cast<uint64_t>(ech), reinterpret_cast<uint64_t>(biais),
               reinterpret_cast<uint64_t>(x), reinterpret_cast<uint64_t>(y), R, C, N, x_bf16};
    return lancer_gemm_mxfp4_lot(&d, 1, R, C, N, espace, erreur, flux);
}

uint64_t gemm_mxfp4_lot_espace(uint32_t colonnes_max, uint32_t n_max, uint32_t nb) {
    return uint64_t(nb) * ((gemm_mxfp4_espace(colonnes_max, n_max) + 255u) & ~uint64_t(255));
}

}  // namespace tb
