// troncons_b200 — y = W x + b on a decoded SoA slot (the reference's gemv_mxfp4 /
// gemv_mxfp4_lot contract, trc-noyaux/noyaux/gemv.cuh:140-161), and the router's f32 GEMV
// (gemv_f32, passe.cuh:104-130, 225-233).
//
// MXFP4: one warp per row (row-centric, no cross-warp reduction), the reduction order of
// mxfp4.cuh, so a slot GEMV gives the bits of the fused path. x is read through L1 (the same
// x for every row) and doubled in registers.
// Router: one block per row, its float4 chunks split in quarters over 4 warps (order at
// k_gemv_f32); x may be f32 or bf16 (converted exactly).
#include <cuda_bf16.h>

#include "commun.cuh"
#include "gemv_groupes.cuh"
#include "mxfp4.cuh"
#include "noyaux.h"

namespace tb {

constexpr uint32_t GEMV_WARPS = 8;

__device__ __forceinline__ void gemv_lignes(const uint8_t* __restrict__ mat, const float* __restrict__ x, float* __restrict__ y,
                                            uint32_t R, uint32_t C, uint32_t ligne0, uint32_t pas) {
    const uint32_t voie = threadIdx.x & 31u;
    const uint32_t B = C / 32u;
    const Disposition d = disposition_matrice(R, C);
    const uint8_t* ech = mat + d.echelles;
    const float* biais = reinterpret_cast<const float*>(mat + d.biais);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    auto x2f4 = [x4](uint32_t i) { return fois2(__ldg(x4 + i)); };
    for (uint32_t r = ligne0; r < R; r += pas) {
        const float t = ligne_segments(mat, ech, x2f4, r, B, voie, nullptr);
        if (voie == 0) y[r] = t + biais[r];
    }
}

__global__ void __launch_bounds__(GEMV_WARPS * 32) k_gemv(const uint8_t* __restrict__ mat, const float* __restrict__ x,
                                                          float* __restrict__ y, uint32_t R, uint32_t C) {
    attendre_amont();
    liberer_aval();
    gemv_lignes(mat, x, y, R, C, blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5), gridDim.x * GEMV_WARPS);
}

__global__ void __launch_bounds__(GEMV_WARPS * 32) k_gemv_lot(const DescGemv* __restrict__ descs) {
    attendre_amont();
    liberer_aval();
    const DescGemv d = descs[blockIdx.y];
    if (d.colonnes % 32u != 0 || d.lignes == 0) return;
    gemv_lignes(reinterpret_cast<const uint8_t*>(d.matrice), reinterpret_cast<const float*>(d.x), reinterpret_cast<float*>(d.y),
                d.lignes, d.colonnes, blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5), gridDim.x * GEMV_WARPS);
}

// The batch of slot GEMVs in row groups (gemv_groupes.cuh) where the shapes allow: blockIdx.y
// is the matrix, its blocks share the matrix's staged 2x, each warp takes row groups
// blockIdx.x * W + warp, + gridDim.x * W. Other shapes take gemv_lignes (the same bits).
__global__ void __launch_bounds__(128, 3) k_gemv_lot_groupes(const DescGemv* __restrict__ descs) {
    extern __shared__ __align__(16) uint8_t dyn[];
    attendre_amont();
    liberer_aval();
    const DescGemv d = descs[blockIdx.y];
    if (d.colonnes % 32u != 0 || d.lignes == 0) return;
    const uint32_t R = d.lignes, C = d.colonnes, B = C / 32u, W = blockDim.x >> 5, warp = threadIdx.x >> 5;
    const uint8_t* mat = reinterpret_cast<const uint8_t*>(d.matrice);
    if (!groupes_possibles(R, B)) {
        gemv_lignes(mat, reinterpret_cast<const float*>(d.x), reinterpret_cast<float*>(d.y), R, C,
                    blockIdx.x * W + warp, gridDim.x * W);
        return;
    }
    float4* x2g = reinterpret_cast<float4*>(dyn);
    charger_x2_groupes(x2g, reinterpret_cast<const float*>(d.x), 0u, C);
    __syncthreads();
    const Disposition dm = disposition_matrice(R, C);
    gemv_groupes<false>(mat, mat + dm.echelles, reinterpret_cast<const float*>(mat + dm.biais), x2g, R, B,
                        reinterpret_cast<float*>(d.y), 0u, blockIdx.x * W + warp, gridDim.x * W);
}

__device__ __forceinline__ float4 charger_x4(const void* x, uint32_t x_bf16, uint32_t c) {
    if (x_bf16) {
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(x) + c);
        return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u), __uint_as_float(v.y << 16),
                           __uint_as_float(v.y & 0xFFFF0000u));
    }
    return __ldg(reinterpret_cast<const float4*>(x) + c);
}

// One block per row, 4 warps: warp q takes the q-th quarter of the row's float4 chunks
// (Q = ceil(C/16) chunks each), lane l the chunks q Q + l, + 32, ... in an fmaf chain (x, y, z, w);
// xor butterfly 16 .. 1 in each warp; y = ((p0 + p1) + (p2 + p3)) + b. Every lane's loads (at
// most 6 float4 for C = 2880) are in flight together.
constexpr uint32_t F32_QUARTS = 4;

__global__ void __launch_bounds__(F32_QUARTS * 32) k_gemv_f32(const float* __restrict__ w, const void* x,
                                                             uint32_t x_bf16, const float* __restrict__ biais,
                                                             float* y, uint32_t R, uint32_t C) {
    __shared__ float parts[F32_QUARTS];
    attendre_amont();
    liberer_aval();
    const uint32_t r = blockIdx.x, voie = threadIdx.x & 31u, q = threadIdx.x >> 5;
    // Token blockIdx.y of a batch: its x and its y.
    x = static_cast<const uint8_t*>(x) + uint64_t(blockIdx.y) * C * (x_bf16 ? 2u : 4u);
    y += uint64_t(blockIdx.y) * R;
    const uint32_t C4 = C / 4u, Q = (C4 + F32_QUARTS - 1u) / F32_QUARTS, c0 = q * Q, c1 = min(C4, c0 + Q);
    const float4* w4 = reinterpret_cast<const float4*>(w) + uint64_t(r) * C4;
    float acc = 0.0f;
#pragma unroll 8
    for (uint32_t c = c0 + voie; c < c1; c += 32u) {
        const float4 a = __ldcs(w4 + c);
        const float4 b = charger_x4(x, x_bf16, c);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
#pragma unroll
    for (int dd = 16; dd > 0; dd >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, dd);
    if (voie == 0) parts[q] = acc;
    __syncthreads();
    if (threadIdx.x == 0 && r < R) {
        const float s = (parts[0] + parts[1]) + (parts[2] + parts[3]);
        y[r] = biais != nullptr ? s + biais[r] : s;
    }
}

cudaError_t lancer_gemv(const void* matrice, const float* x, float* y, uint32_t R, uint32_t C, cudaStream_t flux) {
    const uint32_t blocs = std::min<uint32_t>((R + GEMV_WARPS - 1) / GEMV_WARPS, 65535u);
    return lancer_pdl(k_gemv, dim3(blocs), dim3(GEMV_WARPS * 32), 0, flux, static_cast<const uint8_t*>(matrice), x, y, R, C);
}

uint32_t sms_courant() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return uint32_t(sms);
}

// The batch in row groups: blocks of 4 warps, one row group per warp (the widest 2x staged
// per block: 2x of up to 8,192 columns), the matrix as grid y.
constexpr uint32_t GRP_WARPS = 4;
cudaError_t lancer_gemv_lot(const DescGemv* descs, uint32_t n, uint32_t lignes_max, cudaStream_t flux) {
    const uint32_t smem = x2g_octets(32u * GRP_B_MAX);
    cudaError_t e = assurer_smem(reinterpret_cast<const void*>(k_gemv_lot_groupes), int(smem));
    if (e != cudaSuccess) return e;
    const uint32_t groupes = (lignes_max + GRP_LIGNES - 1) / GRP_LIGNES;
    const uint32_t bx = std::max(1u, (groupes + GRP_WARPS - 1u) / GRP_WARPS);
    return lancer_pdl(k_gemv_lot_groupes, dim3(bx, n, 1), dim3(32u * GRP_WARPS), smem, flux, descs);
}

cudaError_t lancer_gemv_f32(const float* w, const void* x, uint32_t x_bf16, const float* biais, float* y, uint32_t R,
                            uint32_t C, cudaStream_t flux, uint32_t jetons) {
    return lancer_pdl(k_gemv_f32, dim3(R, jetons), dim3(F32_QUARTS * 32), 0, flux, w, x, x_bf16, biais, y, R, C);
}

}  // namespace tb
