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
// Memory: the code words go straight from HBM to registers, 16 bytes per lane and row-block
// (the 8 lanes of a row read 8 neighbouring blocks: 128 contiguous bytes), two column steps
// ahead of their use; shared memory holds only the block's staged 2x, so many warps fit on an SM and
// keep their loads in flight together.
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

__host__ __device__ __forceinline__ uint32_t x2g_octets(uint32_t C) { return (C / 32u) * GRP_X2_PAS * 16u; }

// 2x of x (bf16 or f32, C a multiple of 32) in the grouped layout: for column block b, float4
// k = 0..3 holds (x2[32b + k], x2[32b + 4 + k], x2[32b + 8 + k], x2[32b + 12 + k]) and float4
// 4 + k the same 16 further (the high nibbles' activations): the quads' k-th operands side by side.
__device__ __forceinline__ void charger_x2_groupes(float4* x2g, const void* x, uint32_t bf16, uint32_t C) {
    // Element i of x goes to float (9 b + 4 h + k) * 4 + q of the staged area, b = i / 32,
    // h = (i / 16) % 2, q = (i / 4) % 4, k = i % 4. Each thread loads 8 consecutive elements with
    // 16-byte loads when x is 16-aligned.
    float* d = reinterpret_cast<float*>(x2g);
    auto poser = [d](uint32_t i, float v) {
        const uint32_t b = i >> 5, h = (i >> 4) & 1u, q = (i >> 2) & 3u, k = i & 3u;
        d[(b * GRP_X2_PAS + 4u * h + k) * 4u + q] = 2.0f * v;
    };
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        for (uint32_t t = threadIdx.x; t < C / 8u; t += blockDim.x) {
            const uint32_t i0 = 8u * t;
            if (bf16) {
                const uint4 v = __ldg(static_cast<const uint4*>(x) + t);
                const uint32_t m[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (uint32_t j = 0; j < 4; ++j) {
                    poser(i0 + 2u * j, __uint_as_float(m[j] << 16));
                    poser(i0 + 2u * j + 1u, __uint_as_float(m[j] & 0xFFFF0000u));
                }
            } else {
                const float4 u = __ldg(static_cast<const float4*>(x) + 2u * t);
                const float4 v = __ldg(static_cast<const float4*>(x) + 2u * t + 1u);
                poser(i0, u.x);
                poser(i0 + 1u, u.y);
                poser(i0 + 2u, u.z);
                poser(i0 + 3u, u.w);
                poser(i0 + 4u, v.x);
                poser(i0 + 5u, v.y);
                poser(i0 + 6u, v.z);
                poser(i0 + 7u, v.w);
            }
        }
        return;
    }
    for (uint32_t i = threadIdx.x; i < C; i += blockDim.x)
        poser(i, bf16 ? __uint_as_float(uint32_t(static_cast<const uint16_t*>(x)[i]) << 16) : static_cast<const float*>(x)[i]);
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

// The groups g0, g0 + pas, ... of a matrix (codes: 16 bytes per block, row-major blocks,
// 16-aligned; echelles: one E8M0 byte per block; R rows, B blocks per row, groupes_possibles(R,
// B)), with the block's staged 2x `x2g`. Per row r: parts[r K + k] = the partial of its k-th
// segment (PARTS), or y[r] = fold + bias. MED: `echelles` holds each block's delta byte and
// `medianes` each row's median (the .trc v1.2 scale coding, trc-codec/src/lib.rs:206-212): the
// block's E8M0 scale is (median + delta - 128) mod 256.
template <bool PARTS, bool MED = false>
__device__ inline void gemv_groupes(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ echelles,
                                    const float* __restrict__ biais, const float4* __restrict__ x2g, uint32_t R,
                                    uint32_t B, float* __restrict__ sortie, uint32_t K, uint32_t g0, uint32_t pas,
                                    const uint8_t* __restrict__ medianes = nullptr) {
    const uint32_t voie = threadIdx.x & 31u, a = voie >> 3, g = voie & 7u;
    const uint32_t ngr = R / GRP_LIGNES;
    for (uint32_t gr = g0; gr < ngr; gr += pas) {
        const uint32_t R0 = gr * GRP_LIGNES;
        // Lane (a, g): slot g of rows R0 + a + 4 i; column blocks c, c + 8, ... with
        // (R0 + a) B + c = g (mod 8).
        const uint32_t c0 = (g + 8u - ((R0 + a) * B) % 8u) % 8u;
        float acc[4][2];
        uint32_t cesure[4];  // first column block of each row's second segment (B when none)
        const uint4* ligne_c[4];
        const uint8_t* ligne_e[4];
        uint32_t decal[4];  // MED: the row's median + 128 (mod 256 once added to a delta)
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            acc[i][0] = 0.0f;
            acc[i][1] = 0.0f;
            const uint32_t r = R0 + a + 4u * i;
            const uint32_t b0 = r * B;
            cesure[i] = min(B, (b0 / SEGMENT_BLOCS + 1u) * SEGMENT_BLOCS - b0);
            ligne_c[i] = reinterpret_cast<const uint4*>(codes) + uint64_t(b0);
            ligne_e[i] = echelles + uint64_t(b0);
            decal[i] = MED ? uint32_t(__ldg(medianes + r)) + 128u : 0u;
        }
        // The four rows' blocks of column block b, loaded two column steps ahead of their use:
        // three buffers in turn (the loop is unrolled by three so that they stay in registers).
        struct Pas {
            uint4 w[4];
            uint32_t e[4];
        };
        auto charger = [&](Pas& p, uint32_t b) {
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                p.w[i] = b < B ? __ldg(ligne_c[i] + b) : make_uint4(0, 0, 0, 0);
                p.e[i] = b < B ? uint32_t(__ldg(ligne_e[i] + b)) : 0u;
            }
        };
        auto calculer = [&](const Pas& p, uint32_t b) {
            if (b >= B) return;
            const float4* xb = x2g + b * GRP_X2_PAS;
#pragma unroll
            for (uint32_t i = 0; i < 4; ++i) {
                const float s = somme_bloc(p.w[i], xb);
                const float sc = echelle_e8m0(MED ? ((p.e[i] + decal[i]) & 255u) : p.e[i]);
                if (b < cesure[i])
                    acc[i][0] = fmaf(s, sc, acc[i][0]);
                else
                    acc[i][1] = fmaf(s, sc, acc[i][1]);
            }
        };
        Pas p0, p1, p2;
        charger(p0, c0);
        charger(p1, c0 + 8u);
        for (uint32_t b = c0; b < B; b += 24u) {
            charger(p2, b + 16u);
            calculer(p0, b);
            charger(p0, b + 24u);
            calculer(p1, b + 8u);
            charger(p1, b + 32u);
            calculer(p2, b + 16u);
        }
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
}

}  // namespace tb
