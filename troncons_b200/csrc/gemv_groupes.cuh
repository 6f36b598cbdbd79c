// troncons_b200 — the MXFP4 GEMV of whole rows streamed from HBM (a decoded slot or a raw part's
// CODES_BRUTS / ECHELLES_BRUTES), in groups of 16 rows per warp, with the reduction order of
// mxfp4.cuh: the same bits as ligne_segments and as the fused rANS-decode GEMV.
//
// Why groups: a GEMV reads one 0.53-byte weight from HBM for each 4-byte activation it
// multiplies, so activations re-read from shared memory per weight would cost ~8x the HBM
// traffic in shared-memory bandwidth. Here a lane multiplies the same column block of 2x by the
// blocks of 4 rows: for B (blocks per row) even, rows r and r + 4 put a column block on the same
// quad slot g = (r B + b) mod 8, so lane (a, g) of a warp (a = lane / 8) owns slot g of rows
// R0 + a + 4 i, i = 0..3, and walks the column blocks b = c + 8 t of that slot, holding 2x of one
// block in registers for the four rows.
//
// Memory: each warp stages its group's code bytes (16 rows x B x 16 bytes, contiguous) and
// scales (16 x B bytes) with one bulk copy each (cp.async.bulk, the TMA engine, completion on an
// mbarrier; no multicast) into one of two buffers, and multiplies the previous group from the
// other while that copy is in flight.
//
// Arithmetic per block (the order of mxfp4.cuh): quad q of the block (bytes 4q..4q+3) gives
// p_q = fmaf chain over k = 0..3 of (low nibble of byte 4q+k) x2[32b+4q+k] then (high nibble)
// x2[32b+16+4q+k], from +0, the four quads' chains two by two in f32x2 FMAs (two independent
// IEEE fmas each); s = (p0 + p1) + (p2 + p3); the slot's accumulator for the block's row and
// 256-block segment: acc = fmaf(s, 2^(e-128), acc); per row and segment the 8 slots' tree
// ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7)) (xor shuffles 1, 2, 4 within the lane's
// group of 8); the row's segments folded in order.
#pragma once

#include "commun.cuh"
#include "mxfp4.cuh"

namespace tb {

constexpr uint32_t GRP_LIGNES = 16;        // rows per warp group (4 sub-rows x 4)
constexpr uint32_t GRP_X2_PAS = 9;         // float4 per column block of the staged 2x (8 + 1 pad)
constexpr uint32_t GRP_B_MAX = 256;        // blocks per row: rows span at most two segments

// Whether a matrix of R rows and B blocks per row takes the grouped GEMV.
__host__ __device__ __forceinline__ bool groupes_possibles(uint32_t R, uint32_t B) {
    return B >= 2u && B <= GRP_B_MAX && (B % 2u) == 0 && R % GRP_LIGNES == 0;
}

// Shared bytes of one staging buffer (a group's codes and scales, 16-aligned) and per warp: two
// buffers (the next group's copy lands while the current one is multiplied) and their mbarriers.
__host__ __device__ __forceinline__ uint32_t groupe_tampon(uint32_t B) {
    return GRP_LIGNES * B * 16u + ((GRP_LIGNES * B + 15u) & ~15u);
}
__host__ __device__ __forceinline__ uint32_t groupe_octets_warp(uint32_t B) { return 2u * groupe_tampon(B) + 16u; }
__host__ __device__ __forceinline__ uint32_t x2g_octets(uint32_t C) { return (C / 32u) * GRP_X2_PAS * 16u; }

// Dynamic shared memory of a grouped launch (one block per SM), and the warps whose staging
// areas fit next to the staged 2x of C columns (8 at most; 8 for gpt-oss's 2880).
constexpr uint32_t GRP_SMEM = 220u * 1024u;
__host__ __device__ __forceinline__ uint32_t warps_groupes(uint32_t C) {
    const uint32_t fixe = x2g_octets(C), par = groupe_octets_warp(C / 32u);
    return fixe + par > GRP_SMEM ? 0u : min(8u, (GRP_SMEM - fixe) / par);
}

// 2x of x (bf16 or f32, C a multiple of 32) in the grouped layout: for column block b, float4
// k = 0..3 holds (x2[32b + k], x2[32b + 4 + k], x2[32b + 8 + k], x2[32b + 12 + k]) and float4
// 4 + k the same 16 further (the high nibbles' activations): the quads' k-th operands side by side.
__device__ __forceinline__ void charger_x2_groupes(float4* x2g, const void* x, uint32_t bf16, uint32_t C) {
    for (uint32_t t = threadIdx.x; t < (C / 32u) * 8u; t += blockDim.x) {
        const uint32_t b = t >> 3, f = t & 7u, k = f & 3u, base = 32u * b + (f >= 4u ? 16u : 0u) + k;
        float v[4];
#pragma unroll
        for (uint32_t q = 0; q < 4; ++q) {
            const uint32_t i = base + 4u * q;
            v[q] = 2.0f * (bf16 ? __uint_as_float(uint32_t(static_cast<const uint16_t*>(x)[i]) << 16)
                                : static_cast<const float*>(x)[i]);
        }
        x2g[b * GRP_X2_PAS + f] = make_float4(v[0], v[1], v[2], v[3]);
    }
}

__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t paire(float lo, float hi) {
    uint64_t d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
    return d;
}
__device__ __forceinline__ float2 depaire(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}

// s of one block: codes (16 bytes as 4 words, word q = quad q), 2x of its column block.
__device__ __forceinline__ float somme_bloc(const uint4 w, const float4* __restrict__ xb) {
    float lo[4][4], hi[4][4];
    e2m1_mot(w.x, lo[0], hi[0]);
    e2m1_mot(w.y, lo[1], hi[1]);
    e2m1_mot(w.z, lo[2], hi[2]);
    e2m1_mot(w.w, lo[3], hi[3]);
    uint64_t p01 = 0, p23 = 0;  // +0, +0
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 a = xb[k], b = xb[4 + k];
        p01 = fma2(paire(lo[0][k], lo[1][k]), paire(a.x, a.y), p01);
        p23 = fma2(paire(lo[2][k], lo[3][k]), paire(a.z, a.w), p23);
        p01 = fma2(paire(hi[0][k], hi[1][k]), paire(b.x, b.y), p01);
        p23 = fma2(paire(hi[2][k], hi[3][k]), paire(b.z, b.w), p23);
    }
    const float2 u = depaire(p01), v = depaire(p23);
    return (u.x + u.y) + (v.x + v.y);
}

__device__ __forceinline__ float arbre8_groupe(float a) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, 1);
    a += __shfl_xor_sync(0xFFFFFFFFu, a, 2);
    a += __shfl_xor_sync(0xFFFFFFFFu, a, 4);
    return a;
}

// Bulk copy of n bytes (n and both addresses 16-aligned) into this CTA's shared memory,
// completing on mbarrier `mb` (the caller arms it with the byte count).
__device__ __forceinline__ void copie_bulk(void* dst, const void* src, uint32_t n, uint64_t* mb) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                     adresse_partagee(dst)),
                 "l"(src), "r"(n), "r"(adresse_partagee(mb))
                 : "memory");
}
__device__ __forceinline__ void mbar_attendre_octets(uint64_t* mb, uint32_t n) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared.b64 st, [%0], %1;\n\t}" ::"r"(adresse_partagee(mb)),
                 "r"(n)
                 : "memory");
}

// The groups g0, g0 + pas, ... of a matrix (codes: 16 bytes per block, row-major blocks;
// echelles: one E8M0 byte per block; R rows, B blocks per row, groupes_possibles(R, B)). Each
// warp calls it with its own staging area `zone` (groupe_octets_warp(B) bytes, 16-aligned) and the
// block's staged 2x `x2g`. Per row r: parts[r K + k] = the partial of its k-th segment (PARTS),
// or y[r] = fold + bias. Returns false when a copy's wait gave up (bounded): that group's outputs
// are then NaN.
template <bool PARTS>
__device__ inline bool gemv_groupes(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ echelles,
                                    const float* __restrict__ biais, const float4* __restrict__ x2g, uint32_t R,
                                    uint32_t B, float* __restrict__ sortie, uint32_t K, uint32_t g0, uint32_t pas,
                                    uint8_t* zone) {
    const uint32_t voie = threadIdx.x & 31u, a = voie >> 3, g = voie & 7u;
    const uint32_t octets_c = GRP_LIGNES * B * 16u, octets_e = GRP_LIGNES * B;  // 16 x B: a multiple of 16
    const uint32_t tampon = groupe_tampon(B);
    uint64_t* mb = reinterpret_cast<uint64_t*>(zone + 2u * tampon);  // mb[0], mb[1]
    if (voie == 0) {
        mbar_init(mb, 1u);
        mbar_init(mb + 1, 1u);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    __syncwarp();
    const uint32_t ngr = R / GRP_LIGNES;
    // Lane 0 stages group gr into buffer t (after the previous reads of that buffer, which the
    // caller ordered with __syncwarp, as the copy engine is another proxy).
    auto lancer = [&](uint32_t gr, uint32_t t) {
        if (voie == 0 && gr < ngr) {
            const uint32_t R0 = gr * GRP_LIGNES;
            uint8_t* z = zone + t * tampon;
            asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
            mbar_attendre_octets(mb + t, octets_c + octets_e);
            copie_bulk(z, codes + uint64_t(R0) * B * 16u, octets_c, mb + t);
            copie_bulk(z + octets_c, echelles + uint64_t(R0) * B, octets_e, mb + t);
        }
    };
    lancer(g0, 0u);
    lancer(g0 + pas, 1u);
    uint32_t parite[2] = {0u, 0u};
    uint32_t t = 0;
    for (uint32_t gr = g0; gr < ngr; gr += pas, t ^= 1u) {
        const uint32_t R0 = gr * GRP_LIGNES;
        const uint8_t* zc = zone + t * tampon;
        const uint8_t* ze = zc + octets_c;
        if (!mbar_attendre(mb + t, parite[t])) {
            mbar_attendre(mb + t, parite[t]);        // second bounded waits for the copies in flight
            mbar_attendre(mb + (t ^ 1u), parite[t ^ 1u]);
            // The group's outputs read NaN rather than stale values.
            for (uint32_t i = voie; i < GRP_LIGNES; i += 32u) {
                if (PARTS) {
                    for (uint32_t k = 0; k < K; ++k) sortie[uint64_t(R0 + i) * K + k] = __int_as_float(0x7FC00000);
                } else {
                    sortie[R0 + i] = __int_as_float(0x7FC00000);
                }
            }
            return false;
        }
        parite[t] ^= 1u;
        // Lane (a, g): slot g of rows R0 + a + 4 i; column blocks c, c + 8, ... with
        // (R0 + a) B + c = g (mod 8).
        const uint32_t c0 = (g + 8u - ((R0 + a) * B) % 8u) % 8u;
        float acc[4][2];
        uint32_t cesure[4];  // first column block of each row's second segment (B when none)
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            acc[i][0] = 0.0f;
            acc[i][1] = 0.0f;
            const uint32_t r = R0 + a + 4u * i;
            const uint32_t b0 = r * B;
            cesure[i] = min(B, (b0 / SEGMENT_BLOCS + 1u) * SEGMENT_BLOCS - b0);
        }
        for (uint32_t b = c0; b < B; b += 8u) {
            const float4* xb = x2g + b * GRP_X2_PAS;
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                const uint32_t ligne = a + 4u * i;  // row within the group
                const uint32_t bl = ligne * B + b;
                const uint4 w = *reinterpret_cast<const uint4*>(zc + 16u * bl);
                const float s = somme_bloc(w, xb);
                const float sc = echelle_e8m0(ze[bl]);
                if (b < cesure[i])
                    acc[i][0] = fmaf(s, sc, acc[i][0]);
                else
                    acc[i][1] = fmaf(s, sc, acc[i][1]);
            }
        }
        __syncwarp();  // every lane is done with this buffer before the copy engine refills it
        lancer(gr + 2u * pas, t);
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            const float P0 = arbre8_groupe(acc[i][0]);
            const float P1 = arbre8_groupe(acc[i][1]);
            const uint32_t r = R0 + a + 4u * i;
            const bool deux = cesure[i] < B;
            if (g == 0) {
                if (PARTS) {
                    sortie[uint64_t(r) * K] = P0;
                    if (deux) sortie[uint64_t(r) * K + 1u] = P1;
                } else {
                    sortie[r] = (deux ? P0 + P1 : P0) + biais[r];
                }
            }
        }
    }
    return true;
}

}  // namespace tb
