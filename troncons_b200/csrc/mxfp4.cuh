// troncons_b200 — MXFP4 arithmetic and the fixed reduction order shared by every GEMV path
// (the GEMV of a decoded slot, the fused rANS-decode GEMV, the raw-part GEMV), so that all of
// them give the same bits on the same weights.
//
// Weight value (gemv.cuh:1-12 of the reference): K[c & 7] * 2^(e - 128), K = {0,1,2,3,4,6,8,12}
// signed by bit 3 (the doubled E2M1 magnitudes), e the block's E8M0 byte. Byte i of a 16-byte
// block carries element i (low nibble) and element 16 + i (high nibble). Here the nibbles are
// converted by the hardware (cvt.rn.f16x2.e2m1x2: the E2M1 values {0,.5,1,...,6}) and the
// activation is doubled once (x2 = 2x, exact), so each product E2M1(c) * x2 equals K[c] * x.
//
// Order (f32, fmaf rounds once):
//   p   per lane of a quad (bytes 4q..4q+3 of a block): fmaf chain, k = 0..3, low nibble with
//       x2[32b + 4q + k] then high nibble with x2[32b + 16 + 4q + k], from +0;
//   s   per block: (p0 + p1) + (p2 + p3)  (xor shuffles 1, 2);
//   acc per row, segment and quad slot g = block % 8: fmaf chain of (s, 2^(e-128)) over the
//       row's blocks of the segment (256 blocks = 32 macro-steps of 8 blocks), from +0;
//   P   per row and segment: ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7))  (xor 4, 8, 16);
//   y   = ((P_g0 + P_g0+1) + ...) + bias.
// -0 codes give the same bits as +0: accumulators start at +0 and +0 + -0 = +0.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

namespace tb {

constexpr uint32_t SEGMENT_BLOCS = 256u;   // blocks per reduction segment
constexpr uint32_t SEGMENT_MACRO = 32u;    // macro-steps (8 blocks each) per segment

// The 8 E2M1 values of a 32-bit code word: lo[k] = low nibble of byte k, hi[k] = high nibble.
__device__ __forceinline__ void e2m1_mot(uint32_t mot, float (&lo)[4], float (&hi)[4]) {
    uint32_t h[4];
    asm("{\n\t.reg .b8 a0, a1, a2, a3;\n\t"
        "mov.b32 {a0, a1, a2, a3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 %0, a0;\n\t"
        "cvt.rn.f16x2.e2m1x2 %1, a1;\n\t"
        "cvt.rn.f16x2.e2m1x2 %2, a2;\n\t"
        "cvt.rn.f16x2.e2m1x2 %3, a3;\n\t}"
        : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
        : "r"(mot));
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        lo[k] = __half2float(__ushort_as_half(static_cast<unsigned short>(h[k] & 0xFFFFu)));
        hi[k] = __half2float(__ushort_as_half(static_cast<unsigned short>(h[k] >> 16)));
    }
}

// p of one quad lane: xa = x2[32b + 4q .. +3], xb = x2[32b + 16 + 4q .. +3].
__device__ __forceinline__ float produit_quad(uint32_t mot, const float4 xa, const float4 xb) {
    float lo[4], hi[4];
    e2m1_mot(mot, lo, hi);
    float p = 0.0f;
    p = fmaf(lo[0], xa.x, p);
    p = fmaf(hi[0], xb.x, p);
    p = fmaf(lo[1], xa.y, p);
    p = fmaf(hi[1], xb.y, p);
    p = fmaf(lo[2], xa.z, p);
    p = fmaf(hi[2], xb.z, p);
    p = fmaf(lo[3], xa.w, p);
    p = fmaf(hi[3], xb.w, p);
    return p;
}

// 2^(e - 128) in f32, exact for every e (e = 0, 1: subnormal).
__device__ __forceinline__ float echelle_e8m0(uint32_t e) {
    return __uint_as_float(e >= 2u ? (e - 1u) << 23 : (0x00200000u << e));
}

__device__ __forceinline__ float somme_quad(float p) {
    p += __shfl_xor_sync(0xFFFFFFFFu, p, 1);
    p += __shfl_xor_sync(0xFFFFFFFFu, p, 2);
    return p;
}

__device__ __forceinline__ float arbre8(float a) {
    a += __shfl_xor_sync(0xFFFFFFFFu, a, 4);
    a += __shfl_xor_sync(0xFFFFFFFFu, a, 8);
    a += __shfl_xor_sync(0xFFFFFFFFu, a, 16);
    return a;
}

__device__ __forceinline__ float4 fois2(float4 v) {
    v.x *= 2.0f;
    v.y *= 2.0f;
    v.z *= 2.0f;
    v.w *= 2.0f;
    return v;
}

// Segment partials of row r, row-centric: one warp walks the row's macro-steps (blocks 8m..8m+7,
// quad g = lane / 4 on block 8m + g), so every lane of a quad holds the block's s. `x2f4(i)`
// gives float4 i of 2x. When `parts` is given, lane 0 writes P of the row's k-th segment to
// parts[k]. Returns the fold of the partials (without bias). The row's code words and scales are
// loaded up to 16 macro-steps at a time before any is used (memory-level parallelism).
constexpr uint32_t LIGNE_LOT = 16u;

template <typename X2>
__device__ __forceinline__ float ligne_segments(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ ech,
                                                X2 x2f4, uint32_t r, uint32_t B, uint32_t voie, float* __restrict__ parts) {
    const uint32_t q = voie & 3u, g = voie >> 2;
    const uint64_t b0 = uint64_t(r) * B, b1 = b0 + B;
    const uint64_t ma = b0 >> 3, mb = (b1 - 1) >> 3;
    float acc = 0.0f, total = 0.0f;
    uint64_t seg = ma / SEGMENT_MACRO;
    uint32_t k = 0;
    for (uint64_t mc = ma; mc <= mb; mc += LIGNE_LOT) {
        uint32_t mots[LIGNE_LOT], es[LIGNE_LOT];
#pragma unroll
        for (uint32_t i = 0; i < LIGNE_LOT; ++i) {
            const uint64_t beta = 8u * (mc + i) + g;
            const bool v = mc + i <= mb && beta >= b0 && beta < b1;
            mots[i] = v ? __ldg(reinterpret_cast<const uint32_t*>(codes + 16u * beta) + q) : 0u;
            es[i] = v ? uint32_t(__ldg(ech + beta)) : 0u;
        }
#pragma unroll
        for (uint32_t i = 0; i < LIGNE_LOT; ++i) {
            const uint64_t m = mc + i;
            if (m > mb) break;
            if (m / SEGMENT_MACRO != seg) {
                const float P = arbre8(acc);
                if (parts != nullptr && voie == 0) parts[k] = P;
                total = k == 0 ? P : total + P;
                ++k;
                acc = 0.0f;
                seg = m / SEGMENT_MACRO;
            }
            const uint64_t beta = 8u * m + g;
            const bool valide = beta >= b0 && beta < b1;
            const uint32_t bc = valide ? uint32_t(beta - b0) : 0u;
            float s = produit_quad(mots[i], x2f4(8u * bc + q), x2f4(8u * bc + 4u + q));
            s = somme_quad(s);
            if (valide) acc = fmaf(s, echelle_e8m0(es[i]), acc);
        }
    }
    const float P = arbre8(acc);
    if (parts != nullptr && voie == 0) parts[k] = P;
    return k == 0 ? P : total + P;
}

// ---------------------------------------------------------------- 2x staged in shared memory

// 2x in shared memory, padded: the 8 float4 of 32-column block b (x2[32 b + 4 k .. + 3], k = 0..7)
// at float4 index 12 b + k. A quarter-warp's 8 lanes read one float4 each from two neighbouring
// blocks; 12 float4 (192 bytes) per block put those blocks 16 banks apart, where 8 (128 bytes)
// would put them on the same banks.
constexpr uint32_t X2_PAS = 12;
__host__ __device__ __forceinline__ uint32_t x2_octets(uint32_t C) { return (C / 32u) * X2_PAS * 16u; }
__device__ __forceinline__ uint32_t x2_indice(uint32_t i) { return X2_PAS * (i / 8u) + (i % 8u); }  // float4 i of 2x

// The padded 2x of x (bf16 or f32, C a multiple of 32); 16-byte loads when x is 16-aligned.
__device__ __forceinline__ void charger_x2(float* x2s, const void* x, uint32_t bf16, uint32_t C) {
    float4* d4 = reinterpret_cast<float4*>(x2s);
    if ((reinterpret_cast<uintptr_t>(x) & 15u) == 0) {
        if (bf16) {
            const uint4* s4 = static_cast<const uint4*>(x);
            for (uint32_t t = threadIdx.x; t < C / 8u; t += blockDim.x) {
                const uint4 v = __ldg(s4 + t);
                d4[x2_indice(2u * t)] = make_float4(2.0f * __uint_as_float(v.x << 16), 2.0f * __uint_as_float(v.x & 0xFFFF0000u),
                                                    2.0f * __uint_as_float(v.y << 16), 2.0f * __uint_as_float(v.y & 0xFFFF0000u));
                d4[x2_indice(2u * t + 1u)] = make_float4(2.0f * __uint_as_float(v.z << 16), 2.0f * __uint_as_float(v.z & 0xFFFF0000u),
                                                         2.0f * __uint_as_float(v.w << 16), 2.0f * __uint_as_float(v.w & 0xFFFF0000u));
            }
        } else {
            const float4* s4 = static_cast<const float4*>(x);
            for (uint32_t t = threadIdx.x; t < C / 4u; t += blockDim.x) d4[x2_indice(t)] = fois2(__ldg(s4 + t));
        }
        return;
    }
    for (uint32_t t = threadIdx.x; t < C; t += blockDim.x) {
        const float v = bf16 ? __uint_as_float(uint32_t(static_cast<const uint16_t*>(x)[t]) << 16) : static_cast<const float*>(x)[t];
        x2s[4u * x2_indice(t / 4u) + (t % 4u)] = 2.0f * v;
    }
}

// Fold of a row's segment partials, as ligne_segments folds them.
__device__ __forceinline__ float finir_ligne(const float* __restrict__ parts, uint32_t r, uint32_t B) {
    const uint64_t b0 = uint64_t(r) * B;
    const uint32_t n = uint32_t((b0 + B - 1) / SEGMENT_BLOCS - b0 / SEGMENT_BLOCS) + 1u;
    float t = parts[0];
    for (uint32_t k = 1; k < n; ++k) t = t + parts[k];
    return t;
}

// Partial slots per row for B blocks per row: the most segments a row can span.
__host__ __device__ __forceinline__ uint32_t parts_par_ligne(uint32_t B) { return (B + SEGMENT_BLOCS - 2u) / SEGMENT_BLOCS + 1u; }

}  // namespace tb
