// troncons_b200 — the geometry-1 rANS encoder on the GPU: a `.trc` stream (rans.rs:186-228) of P
// bytes in tiles of N macro-steps, byte for byte what the CPU encoders write (trc-codec
// rans.rs:296-334; the reference bench's coder_g1, banc_k.cu:277-321).
//
// Tiles are independent: one warp per tile walks the tile backwards (macro-steps m, sub-steps
// k = 3..0), lane l encoding byte 4 (32 m + l) + k with the table of its context (the 16-byte
// block's class kappa, or table 0): renormalise when x >= f << 20 (push the low 16 bits), then
// x = (x / f) M + (x mod f) + c. The pushes of one sub-step go in lane order 31 .. 0 (a ballot
// ranks them), onto the tile's stack in scratch memory. A second pass lays out the stream:
// header, tile starts (prefix sum of the tiles' word counts), final lane states, and each tile's
// words as its stack reversed, then zero padding to 16 bytes.
#include "commun.cuh"
#include "noyaux.h"

namespace tb {

constexpr uint32_t CODEUR_WARPS = 8;
constexpr uint32_t CODEUR_TABLES_MAX = 4;

// Scratch of an encode: per tile, a stack of up to 128 N words (one per lane and sub-step),
// the tile's word count, and its 32 final states.
__host__ __device__ __forceinline__ uint64_t pile_mots(uint32_t N) { return 128ull * N; }

__global__ void __launch_bounds__(CODEUR_WARPS * 32) k_coder_tuiles(const uint8_t* __restrict__ src, uint32_t P, uint32_t N,
                                                                  const uint8_t* __restrict__ kappa, uint32_t n_kappa,
                                                                  const uint16_t* __restrict__ freqs, uint32_t n_tables,
                                                                  uint16_t* __restrict__ piles, uint32_t* __restrict__ n_mots,
                                                                  uint32_t* __restrict__ etats, uint32_t* erreur) {
    __shared__ uint32_t F[CODEUR_TABLES_MAX][256], Cc[CODEUR_TABLES_MAX][256];
    attendre_amont();
    liberer_aval();
    for (uint32_t t = threadIdx.x; t < n_tables * 256u; t += blockDim.x) F[t / 256u][t % 256u] = freqs[t];
    __syncthreads();
    if (threadIdx.x < n_tables) {  // cumulative frequencies, one table per thread
        uint32_t c = 0;
        for (uint32_t s = 0; s < 256u; ++s) {
            Cc[threadIdx.x][s] = c;
            c += F[threadIdx.x][s];
        }
    }
    __syncthreads();
    const uint32_t voie = threadIdx.x & 31u;
    const uint32_t n_macro = P / 128u, T = (n_macro + N - 1) / N;
    const uint32_t t = blockIdx.x * CODEUR_WARPS + (threadIdx.x >> 5);
    if (t >= T) return;
    const uint32_t m0 = t * N, m1 = min(m0 + N, n_macro);
    uint16_t* pile = piles + uint64_t(t) * pile_mots(N);
    uint32_t x = L, np = 0, manque = 0;
    const uint32_t dessus = voie == 31u ? 0u : (0xFFFFFFFFu << (voie + 1u));  // lanes above this one
    for (uint32_t m = m1; m-- > m0;) {
        const uint32_t w = m * 32u + voie;
        const uint32_t mot = __ldg(reinterpret_cast<const uint32_t*>(src) + w);
        uint32_t ctx = kappa != nullptr && (w >> 2) < n_kappa ? uint32_t(__ldg(kappa + (w >> 2))) : 0u;
        manque |= ctx >= n_tables ? 1u : 0u;  // a context without a table: an encoding error
        ctx = ctx < n_tables ? ctx : 0u;
#pragma unroll
        for (int k = 3; k >= 0; --k) {
            const uint32_t s = (mot >> (8 * k)) & 0xFFu;
            const uint32_t f = F[ctx][s], c = Cc[ctx][s];
            manque |= f == 0u ? 1u : 0u;
            const uint32_t fs = f == 0u ? 1u : f;
            const bool pousse = uint64_t(x) >= (uint64_t(fs) << 20);
            const uint32_t vote = __ballot_sync(0xFFFFFFFFu, pousse);
            if (pousse) pile[np + __popc(vote & dessus)] = uint16_t(x & 0xFFFFu);
            np += __popc(vote);
            const uint32_t xv = pousse ? x >> 16 : x;
            x = (xv / fs) * M + (xv % fs) + c;
        }
    }
    etats[uint64_t(t) * 32u + voie] = x;
    if (voie == 0) n_mots[t] = np;
    if (__any_sync(0xFFFFFFFFu, manque) && voie == 0) atomicOr(erreur, 1u);
}

// One block: tile starts (prefix sum over the tiles' word counts, in order), the header, the
// starts and the states; the stream's byte length into *octets. Nothing is written when the
// stream would not fit in `capacite` (*octets still says how many bytes it needs).
__global__ void __launch_bounds__(1024) k_flux_tete(uint32_t P, uint32_t N, const uint32_t* __restrict__ n_mots,
                                                    const uint32_t* __restrict__ etats, uint32_t* __restrict__ debuts,
                                                    uint8_t* __restrict__ sortie, uint64_t capacite, uint64_t* octets,
                                                    const uint32_t* erreur) {
    __shared__ uint32_t part[1024];
    __shared__ uint32_t base;
    attendre_amont();
    liberer_aval();
    const uint32_t T = (P / 128u + N - 1) / N;
    // exclusive scan, 1024 tiles at a time
    if (threadIdx.x == 0) base = 0;
    __syncthreads();
    for (uint32_t t0 = 0; t0 < T; t0 += 1024u) {
        const uint32_t t = t0 + threadIdx.x;
        const uint32_t v = t < T ? n_mots[t] : 0u;
        part[threadIdx.x] = v;
        __syncthreads();
        for (uint32_t d = 1; d < 1024u; d <<= 1) {
            const uint32_t a = threadIdx.x >= d ? part[threadIdx.x - d] : 0u;
            __syncthreads();
            part[threadIdx.x] += a;
            __syncthreads();
        }
        if (t < T) debuts[t] = base + part[threadIdx.x] - v;
        __syncthreads();
        if (threadIdx.x == 1023u) base += part[1023];
        __syncthreads();
    }
    const uint32_t W = base;
    const uint64_t lg = (16ull + 132ull * T + 2ull * W + 15ull) & ~15ull;
    if (threadIdx.x == 0) *octets = (*erreur != 0u) ? 0ull : lg;
    if (lg > capacite || *erreur != 0u) return;
    if (threadIdx.x == 0) {
        uint32_t* h = reinterpret_cast<uint32_t*>(sortie);
        h[0] = P;
        h[1] = (N & 0xFFFFu) | (1u << 16);  // N, geometry 1, reserved 0
        h[2] = T;
        h[3] = W;
    }
    uint32_t* d = reinterpret_cast<uint32_t*>(sortie + 16);
    for (uint32_t t = threadIdx.x; t < T; t += blockDim.x) d[t] = debuts[t];
    uint32_t* e = reinterpret_cast<uint32_t*>(sortie + 16 + 4ull * T);
    for (uint32_t i = threadIdx.x; i < 32u * T; i += blockDim.x) e[i] = etats[i];
}

// The words: tile t's stack reversed at its start; the padding zeroed.
__global__ void __launch_bounds__(256) k_flux_mots(uint32_t P, uint32_t N, const uint16_t* __restrict__ piles,
                                                   const uint32_t* __restrict__ n_mots, const uint32_t* __restrict__ debuts,
                                                   uint8_t* __restrict__ sortie, uint64_t capacite, const uint64_t* octets) {
    attendre_amont();
    liberer_aval();
    const uint32_t T = (P / 128u + N - 1) / N;
    const uint64_t lg = *octets;
    if (lg == 0 || lg > capacite) return;
    const uint32_t t = blockIdx.y;
    if (t >= T) return;
    const uint32_t n = n_mots[t];
    uint16_t* mots = reinterpret_cast<uint16_t*>(sortie + 16 + 132ull * T) + debuts[t];
    const uint16_t* pile = piles + uint64_t(t) * pile_mots(N);
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) mots[j] = pile[n - 1u - j];
    if (t == T - 1 && blockIdx.x == 0) {
        const uint64_t fin = 16ull + 132ull * T + 2ull * (debuts[t] + n);
        for (uint64_t o = fin + threadIdx.x; o < lg; o += blockDim.x) sortie[o] = 0;
    }
}

uint64_t coder_flux_espace(uint32_t P, uint32_t N) {
    const uint64_t T = (uint64_t(P) / 128u + N - 1) / N;
    return ((T * pile_mots(N) * 2u + 255u) & ~uint64_t(255)) + ((T * 4u + 255u) & ~uint64_t(255)) * 2u +
           ((T * 128u + 255u) & ~uint64_t(255)) + 256u;
}

cudaError_t lancer_coder_flux(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, uint32_t n_kappa,
                              const uint16_t* freqs, uint32_t n_tables, uint8_t* sortie, uint64_t capacite, uint64_t* octets,
                              uint8_t* espace, cudaStream_t flux) {
    const uint32_t T = (P / 128u + N - 1) / N;
    uint8_t* p = espace;
    uint16_t* piles = reinterpret_cast<uint16_t*>(p);
    p += (uint64_t(T) * pile_mots(N) * 2u + 255u) & ~uint64_t(255);
    uint32_t* n_mots = reinterpret_cast<uint32_t*>(p);
    p += (uint64_t(T) * 4u + 255u) & ~uint64_t(255);
    uint32_t* debuts = reinterpret_cast<uint32_t*>(p);
    p += (uint64_t(T) * 4u + 255u) & ~uint64_t(255);
    uint32_t* etats = reinterpret_cast<uint32_t*>(p);
    p += (uint64_t(T) * 128u + 255u) & ~uint64_t(255);
    uint32_t* erreur = reinterpret_cast<uint32_t*>(p);
    cudaError_t e = cudaMemsetAsync(erreur, 0, 4, flux);
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_coder_tuiles, dim3((T + CODEUR_WARPS - 1) / CODEUR_WARPS), dim3(CODEUR_WARPS * 32), 0, flux, src, P, N,
                   kappa, n_kappa, freqs, n_tables, piles, n_mots, etats, erreur);
    if (e != cudaSuccess) return e;
    e = lancer_pdl(k_flux_tete, dim3(1), dim3(1024), 0, flux, P, N, static_cast<const uint32_t*>(n_mots),
                   static_cast<const uint32_t*>(etats), debuts, sortie, capacite, octets, static_cast<const uint32_t*>(erreur));
    if (e != cudaSuccess) return e;
    return lancer_pdl(k_flux_mots, dim3(4, T), dim3(256), 0, flux, P, N, static_cast<const uint16_t*>(piles),
                      static_cast<const uint32_t*>(n_mots), static_cast<const uint32_t*>(debuts), sortie, capacite,
                      static_cast<const uint64_t*>(octets));
}

}  // namespace tb
