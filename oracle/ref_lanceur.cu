// TEST INFRASTRUCTURE — C entry points for the reference's own CUDA kernels.
//
// The reference's kernels (moteur/crates/trc-noyaux/noyaux/noyaux.cu and the headers it
// includes) are compiled unchanged for sm_100a from the reference checkout by oracle/Makefile;
// this file only launches them with the reference's grids (trc-noyaux/src/abi.rs:130-184,
// noyaux/src/lib.rs:118-496), so the tests can compare troncons_b200 against the reference's
// decoder on the same bytes. Nothing of the reference is copied here.
#include "noyaux.cu"

#include <cuda_runtime.h>

namespace {
uint32_t tuiles(uint64_t octets) { return (uint32_t)(((octets + 127) / 128 + 255) / 256); }
uint64_t blocs(const trc::DimsExpert& d, int j) { return (uint64_t)d.lignes[j] * (d.colonnes[j] / 32); }
trc::DimsExpert dims_de(const uint32_t* d6) {
    trc::DimsExpert d;
    for (int j = 0; j < 3; ++j) {
        d.lignes[j] = d6[j];
        d.colonnes[j] = d6[3 + j];
    }
    return d;
}
}  // namespace

extern "C" int ref_decoder_expert(const void* partie, void* emplacement, const uint32_t* luts, const uint32_t* dims6,
                                  uint32_t* controle, void* flux) {
    const trc::DimsExpert d = dims_de(dims6);
    uint32_t td = 1, tc = 1;
    for (int j = 0; j < 3; ++j) {
        td = td > tuiles(blocs(d, j)) ? td : tuiles(blocs(d, j));
        tc = tc > tuiles(16 * blocs(d, j)) ? tc : tuiles(16 * blocs(d, j));
    }
    cudaStream_t s = (cudaStream_t)flux;
    decoder_echelles<<<dim3((td + 3) / 4, 3, 1), 128, 0, s>>>((const uint8_t*)partie, (uint8_t*)emplacement, luts, d, controle);
    decoder_codes<<<dim3((tc + 7) / 8, 3, 1), 256, 0, s>>>((const uint8_t*)partie, (uint8_t*)emplacement, luts, d, controle);
    return (int)cudaGetLastError();
}

extern "C" int ref_copier_brut(const void* partie, void* emplacement, const uint32_t* dims6, uint32_t* controle, void* flux) {
    const trc::DimsExpert d = dims_de(dims6);
    uint64_t n = 1;
    for (int j = 0; j < 3; ++j) n = n > blocs(d, j) ? n : blocs(d, j);
    uint32_t g = (uint32_t)((n + 255) / 256);
    g = g < 1 ? 1 : (g > 96 ? 96 : g);
    copier_brut<<<dim3(g, 3, 1), 256, 0, (cudaStream_t)flux>>>((const uint8_t*)partie, (uint8_t*)emplacement, d, controle);
    return (int)cudaGetLastError();
}

extern "C" int ref_gemv(const void* matrice, const float* x, float* y, uint32_t R, uint32_t C, void* flux) {
    gemv_mxfp4<<<(R + 31) / 32, 256, 0, (cudaStream_t)flux>>>((const uint8_t*)matrice, x, y, R, C);
    return (int)cudaGetLastError();
}

extern "C" int ref_gemv_lot(const void* descs, uint32_t n, uint32_t lignes_max, void* flux) {
    gemv_mxfp4_lot<<<dim3((lignes_max + 31) / 32, n, 1), 256, 0, (cudaStream_t)flux>>>((const trc::DescGemv*)descs);
    return (int)cudaGetLastError();
}

extern "C" int ref_decoder_lot(const void* descs, uint32_t n, const uint32_t* dims6, void* flux) {
    const trc::DimsExpert d = dims_de(dims6);
    uint32_t td = 1, tc = 1;
    for (int j = 0; j < 3; ++j) {
        td = td > tuiles(blocs(d, j)) ? td : tuiles(blocs(d, j));
        tc = tc > tuiles(16 * blocs(d, j)) ? tc : tuiles(16 * blocs(d, j));
    }
    cudaStream_t s = (cudaStream_t)flux;
    decoder_echelles_lot<<<dim3((td + 3) / 4, 3, n), 128, 0, s>>>((const trc::DescDecodage*)descs, d);
    decoder_codes_lot<<<dim3((tc + 7) / 8, 3, n), 256, 0, s>>>((const trc::DescDecodage*)descs, d);
    return (int)cudaGetLastError();
}

extern "C" int ref_gemv_f32(const float* W, const float* x, const float* biais, float* y, uint32_t R, uint32_t C, void* flux) {
    gemv_f32<<<(R + 31) / 32, 256, 0, (cudaStream_t)flux>>>(W, x, biais, y, R, C);
    return (int)cudaGetLastError();
}

extern "C" int ref_routeur_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices, float* poids, void* flux) {
    routeur_topk<<<1, 32, 0, (cudaStream_t)flux>>>(logits, E, k, indices, poids, nullptr, 0);
    return (int)cudaGetLastError();
}

extern "C" int ref_swiglu(const float* g, const float* u, float* y, uint32_t n, void* flux) {
    swiglu_oai<<<(n + 255) / 256, 256, 0, (cudaStream_t)flux>>>(g, u, y, n);
    return (int)cudaGetLastError();
}

extern "C" int ref_combiner(float* residu, const float* sorties, uint32_t pas, const float* poids, uint32_t n, uint32_t d,
                            void* flux) {
    combiner<<<(d + 255) / 256, 256, 0, (cudaStream_t)flux>>>(residu, sorties, pas, poids, n, d);
    return (int)cudaGetLastError();
}

// ---- the attention side (passe.cuh:222-371), with the reference's grids (lib.rs:291-381)

extern "C" int ref_gemv_q8_0(const void* W, const float* x, const float* biais, float* y, uint32_t R, uint32_t C,
                             void* flux) {
    gemv_q8_0<<<(R + 31) / 32, 256, 0, (cudaStream_t)flux>>>((const uint8_t*)W, x, biais, y, R, C);
    return (int)cudaGetLastError();
}

extern "C" int ref_rmsnorm(const float* x, const float* w, float* y, uint32_t n, uint32_t lignes, float eps, void* flux) {
    rmsnorm<<<lignes, 256, 0, (cudaStream_t)flux>>>(x, w, y, n, eps);
    return (int)cudaGetLastError();
}

extern "C" int ref_rope_yarn(float* q, float* k, uint32_t tetes_q, uint32_t tetes_k, uint32_t position,
                             const trc::ParamsRope* p, void* flux) {
    rope_yarn<<<tetes_q + tetes_k, p->dim_tete / 2, 0, (cudaStream_t)flux>>>(q, k, tetes_q, tetes_k, position, *p);
    return (int)cudaGetLastError();
}

extern "C" int ref_ecrire_kv(const float* k, const float* v, unsigned short* ck, unsigned short* cv, uint32_t dkv,
                             uint32_t case_kv, void* flux) {
    ecrire_kv<<<(dkv + 255) / 256, 256, 0, (cudaStream_t)flux>>>(k, v, ck, cv, dkv, case_kv);
    return (int)cudaGetLastError();
}

extern "C" int ref_attention(const float* q, const unsigned short* ck, const unsigned short* cv, const float* puits,
                             float* sortie, const trc::ParamsAttention* p, void* flux) {
    attention<<<p->tetes, 256, 4 * (p->fin - p->debut), (cudaStream_t)flux>>>(q, ck, cv, puits, sortie, *p);
    return (int)cudaGetLastError();
}
