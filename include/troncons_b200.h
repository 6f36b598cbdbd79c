/*
 * troncons_b200 — the C-ABI of the B200 (sm_100a) kernels for troncons' hot path: on-GPU rANS
 * decoding of `.trc` v1.x MXFP4 expert parts, fused into the MoE expert GEMV.
 *
 * This is the drop-in boundary for the reference's kernel contract (crate trc-noyaux, struct
 * `Noyaux`, moteur/crates/trc-noyaux/src/lib.rs): the same structs, byte for byte, the same
 * argument meaning and the same error behaviour. A Rust host binds it with `extern "C"`
 * declarations of these functions and `#[repr(C)]` twins of these structs. Every launch is asynchronous on the caller's stream
 * (`flux`, a cudaStream_t; NULL is the legacy default stream). The caller owns every device
 * buffer; the library allocates nothing on the device.
 *
 * Status codes: TRC_OK, TRC_ERR_USAGE (a size, alignment or shape the reference's host wrapper
 * also refuses, noyaux/src/lib.rs:70-72 `Erreur::Usage`; nothing was launched), TRC_ERR_CUDA (a
 * launch error). `trc_derniere_erreur()` gives the message of the calling thread's last error.
 *
 * Device-side integrity (commun.cuh:36-44 of the reference): kernels never trap. `controle` is a
 * u32[4] the caller zeroes before a decode; after it, [0] counts rANS lanes whose final state is
 * not L, [1] counts format errors (bad magic, missing stream, inconsistent sizes), [2] counts
 * tiles that did not consume exactly their words. Any non-zero counter is a fatal, named error
 * for the caller (trc-ordo/src/lib.rs:1292-1300). Words read past the end of a tile read as 0,
 * as in the normative CPU decoder (trc-codec/src/rans.rs:427-436).
 */
#ifndef TRONCONS_B200_H
#define TRONCONS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRC_OK 0
#define TRC_ERR_USAGE 1
#define TRC_ERR_CUDA 2

/* Rows/columns of an expert's three matrices (gate j=0, up j=1, down j=2): 24 bytes, align 4.
 * Same layout as `abi::DimsExpert` (trc-noyaux/src/abi.rs:8-13; noyaux/commun.cuh:49-52). */
typedef struct trc_dims_expert {
    uint32_t lignes[3];
    uint32_t colonnes[3];
} trc_dims_expert;

/* One product of a GEMV batch: 32 bytes. Same layout as `abi::DescGemv` (abi.rs:16-27). */
typedef struct trc_desc_gemv {
    uint64_t matrice; /* device address of the matrix in a slot (its codes; multiple of 256) */
    uint64_t x;       /* device address of x, f32[colonnes] (multiple of 16) */
    uint64_t y;       /* device address of y, f32[lignes] */
    uint32_t lignes;
    uint32_t colonnes;
} trc_desc_gemv;

/* One expert of a decode batch: 32 bytes. Same layout as `abi::DescDecodage` (abi.rs:32-53). */
typedef struct trc_desc_decodage {
    uint64_t partie;      /* level-0 part as read from the file (16-byte aligned) */
    uint64_t emplacement; /* SoA slot (multiple of 256) */
    uint64_t luts;        /* the layer's LUTs, u32[3][4][4096] */
    uint64_t controle;    /* u32[4], zeroed by the caller */
} trc_desc_decodage;

/* Message of the calling thread's last error ("" when none). */
const char* trc_derniere_erreur(void);

/* Bytes of an expert slot: the SoA layout of abi.rs:69-122 (codes, scales at al256, biases at
 * al256, matrix stride al256), summed over the three matrices. 13,254,144 for gpt-oss. */
uint64_t trc_taille_emplacement(const trc_dims_expert* dims);

/* ---------------------------------------------------------------- the reference's contract */

/* Decodes a level-0 v1.0/v1.2 part (MEDIANES, BIAIS, DELTA, CODES_CTX of the three matrices)
 * into an SoA slot. Replaces `Noyaux::decoder_expert` / `decoder_expert_grilles`
 * (trc-noyaux/src/lib.rs:118-181). `luts`: the layer's u32[3][4][4096] (>= 196,608 bytes; see
 * trc_luts_couche). Slot 256-aligned and >= trc_taille_emplacement; part 16-aligned, >= 64 B;
 * controle >= 16 B. Any tile size N is accepted. */
int trc_decoder_expert(const void* partie, size_t partie_octets, void* emplacement, size_t emplacement_octets,
                       const uint32_t* luts, size_t luts_octets, const trc_dims_expert* dims, uint32_t* controle,
                       size_t controle_octets, void* flux);

/* n experts of the same dimensions in one launch; `descs`: device trc_desc_decodage[n].
 * Expert by expert, the same bytes and counters as trc_decoder_expert. Replaces
 * `Noyaux::decoder_lot` (lib.rs:190-206). */
int trc_decoder_lot(const trc_desc_decodage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims,
                    void* flux);

/* Raw part (file flag bit 2: ECHELLES_BRUTES, CODES_BRUTS, BIAIS) into the same slot layout.
 * Replaces `Noyaux::copier_brut` (lib.rs:210-235). controle[1] counts format errors. */
int trc_copier_brut(const void* partie, size_t partie_octets, void* emplacement, size_t emplacement_octets,
                    const trc_dims_expert* dims, uint32_t* controle, size_t controle_octets, void* flux);

/* y = W x + b for one matrix of a slot (`matrice` = its codes). x f32[colonnes], 16-aligned;
 * y f32[lignes]. Replaces `Noyaux::gemv` (lib.rs:239-262). The reduction order is fixed by the
 * shape only: the same bits as the fused path on the same weights. */
int trc_gemv(const void* matrice, size_t matrice_octets, const float* x, size_t x_octets, float* y, size_t y_octets,
             uint32_t lignes, uint32_t colonnes, void* flux);

/* n independent products (`descs`: device trc_desc_gemv[n]); lignes_max bounds their rows.
 * Product by product, the same bits as trc_gemv. Replaces `Noyaux::gemv_lot` (lib.rs:274-283). */
int trc_gemv_lot(const trc_desc_gemv* descs, size_t descs_octets, uint32_t n, uint32_t lignes_max, void* flux);

/* y = W x (+ b), W f32 row-major [lignes][colonnes] (16-aligned, colonnes % 4 == 0): the router
 * logits. `biais` may be NULL. Replaces `Noyaux::gemv_f32` (lib.rs:307-319). */
int trc_gemv_f32(const float* w, size_t w_octets, const float* x, size_t x_octets, const float* biais,
                 size_t biais_octets, float* y, size_t y_octets, uint32_t lignes, uint32_t colonnes, void* flux);

/* Top-k of `experts` logits (value decreasing, then index increasing; NaN never chosen),
 * weights = softmax of the k chosen, in f64, rounded to f32. experts <= 256, k <= 8. If `boite`
 * (a device address of host-mapped memory) is not 0, words 1..k receive the indices, words
 * k+1..2k the weights' bits, then word 0 `sequence`, written last after a system fence.
 * Replaces `Noyaux::routeur_topk` (lib.rs:418-430; passe.cuh:455-514). */
int trc_routeur_topk(const float* logits, size_t logits_octets, uint32_t experts, uint32_t k, uint32_t* indices,
                     size_t indices_octets, float* poids, size_t poids_octets, uint64_t boite, uint32_t sequence,
                     void* flux);

/* Clamped SwiGLU of gpt-oss on n pairs, in f64 rounded once to f32:
 * g <- min(g, 7); u <- clamp(u, -7, 7); y = g * sigma(1.702 g) * (u + 1).
 * Replaces `Noyaux::swiglu_oai` (lib.rs:451-458; passe.cuh:598-605). */
int trc_swiglu_oai(const float* g, size_t g_octets, const float* u, size_t u_octets, float* y, size_t y_octets,
                   uint32_t n, void* flux);

/* residu[i] += ((w0 s0[i] + w1 s1[i]) + w2 s2[i]) + ..., j = 0..n-1 in order, products and sums
 * rounded separately (no FMA); s_j = sorties + j*pas floats; `poids` NULL means weights 1.
 * Replaces `Noyaux::combiner` (lib.rs:463-475; passe.cuh:611-622). */
int trc_combiner(float* residu, size_t residu_octets, const float* sorties, size_t sorties_octets, uint32_t pas,
                 const float* poids, size_t poids_octets, uint32_t n, uint32_t d, void* flux);

/* ---------------------------------------------------------------- attention side of a layer */

/* YaRN parameters, 48 bytes, the layout of `abi::ParamsRope` (trc-noyaux/src/abi.rs:228-249):
 * gpt-oss: base 150000, facteur 32, ctx_origine 4096, beta_rapide 32, beta_lent 1, dim_tete 64. */
typedef struct trc_params_rope {
    double base;        /* theta */
    double facteur;     /* s */
    double ctx_origine; /* L0 */
    double beta_rapide;
    double beta_lent;
    uint32_t dim_tete;  /* d (even, <= 128) */
    uint32_t variante;  /* 0: OpenAI's ramp ends; 1: llama.cpp's rounded ends */
} trc_params_rope;

/* Attention of one position, 32 bytes, the layout of `abi::ParamsAttention` (abi.rs:254-290). */
typedef struct trc_params_attention {
    uint32_t tetes;     /* query heads (64) */
    uint32_t tetes_kv;  /* key / value heads (8) */
    uint32_t dim_tete;  /* 64 (the only value accepted) */
    uint32_t debut;     /* first position read */
    uint32_t fin;       /* current position + 1 */
    uint32_t anneau;    /* 0: full cache (case = position); else case = position mod anneau */
    float echelle;      /* 1/sqrt(d) */
    uint32_t reserve;
} trc_params_attention;

/* y = W x (+ b), W Q8_0 (ggml blocks of 34 bytes: f16 d, 32 x i8), rows of colonnes/32 blocks,
 * W 16-aligned; x f32 16-aligned; `biais` may be NULL. Replaces `Noyaux::gemv_q8_0`
 * (lib.rs:291-305; passe.cuh:57-97, 222-231), bit for bit: per lane l, blocks l, l + 32, ...;
 * in a block an fmaf chain over the 32 codes, then fmaf(d, s, acc); xor butterfly; + b. */
int trc_gemv_q8_0(const void* w, size_t w_octets, const float* x, size_t x_octets, const float* biais,
                  size_t biais_octets, float* y, size_t y_octets, uint32_t lignes, uint32_t colonnes, void* flux);

/* RMSNorm of `lignes` vectors of n: y = x w / sqrt(sum x^2 / n + eps), sums in f64 (fixed tree
 * over 256 threads), y rounded once; y may be x. Replaces `Noyaux::rmsnorm` (lib.rs:322-330). */
int trc_rmsnorm(const float* x, size_t x_octets, const float* w, size_t w_octets, float* y, size_t y_octets, uint32_t n,
                uint32_t lignes, float eps, void* flux);

/* YaRN rotation (NEOX halves) of q (tetes_q heads) and k (tetes_k heads) in place at `position`,
 * angle, sine, cosine and rotation in f64. Replaces `Noyaux::rope_yarn` (lib.rs:334-345). */
int trc_rope_yarn(float* q, size_t q_octets, float* k, size_t k_octets, uint32_t tetes_q, uint32_t tetes_k,
                  uint32_t position, const trc_params_rope* p, void* flux);

/* k, v (f32[dkv]) into case `case_kv` of a layer's f16 caches ([case][kv head][d], round to
 * nearest even). Replaces `Noyaux::ecrire_kv` (lib.rs:348-358). */
int trc_ecrire_kv(const float* k, size_t k_octets, const float* v, size_t v_octets, uint16_t* cache_k,
                  size_t cache_k_octets, uint16_t* cache_v, size_t cache_v_octets, uint32_t dkv, uint32_t case_kv,
                  void* flux);

/* Decode attention of one position, every query head, over the cases `p` describes, the head's
 * sink (`puits` f32[tetes]) in the softmax's denominator; sortie f32[tetes * 64]. At most 8,192
 * positions. Replaces `Noyaux::attention` (lib.rs:362-380; passe.cuh:316-371). */
int trc_attention(const float* q, size_t q_octets, const uint16_t* cache_k, size_t cache_k_octets, const uint16_t* cache_v,
                  size_t cache_v_octets, const float* puits, size_t puits_octets, float* sortie, size_t sortie_octets,
                  const trc_params_attention* p, void* flux);

/* ---------------------------------------------------------------- host helpers (no device) */

/* Normalises counts to 12-bit frequencies summing to 4096 (trc-codec/src/rans.rs:83-127);
 * geometrie 1: 256 symbols, 2: 16 symbols. */
int trc_table_depuis_comptes(const uint64_t* comptes, uint32_t geometrie, uint16_t* freq);

/* Geometry-1 LUT of 256 frequencies summing to 4096: lut[i] = s | (f-1) << 8 | (i - c) << 20.
 * Replaces `abi::lut_geometrie1` (abi.rs:187-205). */
int trc_lut_geometrie1(const uint16_t* freq, uint32_t* lut);

/* The layer's LUTs in the kernels' layout (abi.rs:207-221): for matrix j, [j][0] DELTA,
 * [j][1+k] CODES_CTX of scale class k. freqs: u16[3][4][256]; presentes[3][4]: 0 for a table
 * the file lacks (an all-zero LUT, never read by a correct stream). luts: u32[3][4][4096]. */
int trc_luts_couche(const uint16_t* freqs, const uint8_t* presentes, uint32_t* luts);

/* ---------------------------------------------------------------- the encoder (trc-codeur) */

/* Adds one matrix's symbols to a layer's counts u64[4][256] ([0] DELTA, [1+k] CODES_CTX class
 * k; padding counted): preparer_matrice_avec + ComptesMatrice::ajouter
 * (trc-codec/src/lib.rs:348-401). blocs: R*B 17-byte MXFP4 blocks [e, qs x 16] in beta order. */
int trc_comptes_matrice(const uint8_t* blocs, uint32_t lignes, uint32_t blocs_par_ligne, int canonique,
                        uint64_t* comptes);

/* Encodes one expert into a level-0 part (12 streams: MEDIANES, BIAIS, DELTA, CODES_CTX per
 * matrix), the part trc-codeur writes (bins/trc-codeur/src/coder.rs:243-313 with
 * trc-codec/src/lib.rs:417-428 and trc-format/src/lib.rs:882-908). blocs[j]: the matrix's R*B
 * 17-byte blocks; biais[j]: f32[R] bytes; freqs: u16[3][4][256] (the layer's tables);
 * canonique: v1.2 (nibble 8 folded to 0). n_delta / n_codes: macro-steps per tile (256 is
 * what trc-codeur writes). Returns the part length (a multiple of 4096) and writes it into
 * `sortie` when `capacite` suffices; returns -1 on bad input. *utiles receives the useful bytes. */
int64_t trc_coder_partie(const uint8_t* const* blocs, const uint8_t* const* biais, const trc_dims_expert* dims,
                         const uint16_t* freqs, int canonique, uint16_t couche, uint16_t expert, uint32_t n_delta,
                         uint32_t n_codes, uint8_t* sortie, size_t capacite, uint32_t* utiles);

/* The raw part of the same expert (file flag bit 2: 9 streams ECHELLES_BRUTES, CODES_BRUTS,
 * BIAIS per matrix; trc-codec/src/lib.rs:432-445). Origin bytes, not canonicalised. */
int64_t trc_coder_partie_brute(const uint8_t* const* blocs, const uint8_t* const* biais,
                               const trc_dims_expert* dims, uint16_t couche, uint16_t expert, uint8_t* sortie,
                               size_t capacite, uint32_t* utiles);

/* Seeded synthetic MXFP4 matrices: per row sigma = 0.02 * exp(0.3 N(0,1)), weights N(0, sigma),
 * per 32-block E8M0 = floor(log2 max|w|) - 2 (+127), E2M1 round-to-nearest-even with the sign
 * kept (so -0 codes exist, as in gpt-oss's GGUF), biases N(0, 0.01) rounded to bf16 and stored
 * as f32. Matrices premier .. premier + n - 1 of R x C, each drawn from the stream (`graine`,
 * matrix index, row) so a matrix does not depend on which others are drawn with it; blocs:
 * n*R*(C/32)*17 bytes, biais: n*R floats. Runs on up to `fils` host threads (0: all). */
int trc_synth_matrices(uint64_t graine, uint32_t lignes, uint32_t colonnes, uint32_t premier, uint32_t n,
                       uint8_t* blocs, float* biais, int fils);

/* ---------------------------------------------------------------- encoder on the GPU */

/* Scratch bytes of trc_coder_flux_gpu for P source bytes in tiles of N macro-steps. */
uint64_t trc_coder_flux_gpu_espace(uint32_t P, uint32_t N);

/* One geometry-1 rANS stream of the P bytes at `src` (device, P a multiple of 128, 4-aligned) in
 * tiles of N macro-steps, on the GPU: byte for byte what trc-codec's coder writes
 * (rans.rs:296-334). Table of byte n: kappa[n / 16] when `kappa` (device u8[n_kappa]) is given
 * and n / 16 < n_kappa, else 0; `freqs`: device u16[n_tables][256] (n_tables 1..4), each summing
 * to 4096. The stream goes to `sortie` (device, 16-aligned) if it fits in `capacite` bytes;
 * *octets (device u64) receives its size (0 when a byte has no slot in its table or its context
 * has no table). `espace`: device scratch of trc_coder_flux_gpu_espace bytes, 256-aligned.
 * Asynchronous on `flux`; the caller reads *octets after synchronising. */
int trc_coder_flux_gpu(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, uint32_t n_kappa,
                       const uint16_t* freqs, uint32_t n_tables, uint8_t* sortie, size_t capacite, uint64_t* octets,
                       void* espace, size_t espace_octets, void* flux);

/* One expert of a GPU encode batch: 72 bytes, in device memory. */
typedef struct trc_desc_codage {
    uint64_t blocs[3]; /* device: matrix j's R*B 17-byte MXFP4 blocks [e, qs x 16], beta order */
    uint64_t biais[3]; /* device: matrix j's f32[R] biases (4-aligned) */
    uint64_t sortie;   /* device: the part (16-aligned) */
    uint64_t capacite; /* bytes available at sortie */
    uint32_t expert;   /* the expert number in the part header */
    uint32_t reserve;  /* 0 */
} trc_desc_codage;

/* Scratch bytes of trc_coder_parties_gpu for n experts of shape `dims`. */
uint64_t trc_coder_parties_gpu_espace(const trc_dims_expert* dims, uint32_t n, uint32_t n_delta, uint32_t n_codes);

/* The level-0 parts of n experts on the GPU: per expert the part trc_coder_partie writes, byte for
 * byte (coder.rs:243-313, trc-codec lib.rs:348-428, trc-format lib.rs:882-908). freqs: device
 * u16[3][4][256], the layer's tables; octets: device u64[2n], [2e] the part's length (a multiple
 * of 4096; 0 when a symbol has no slot in its table), [2e + 1] its useful bytes. Expert e's part
 * is written at descs[e].sortie only when its length fits descs[e].capacite (zeros included: the
 * whole length is written). espace: device scratch of trc_coder_parties_gpu_espace bytes,
 * 256-aligned. Asynchronous on `flux`. */
int trc_coder_parties_gpu(const trc_desc_codage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims,
                          const uint16_t* freqs, int canonique, uint16_t couche, uint32_t n_delta, uint32_t n_codes,
                          uint64_t* octets, size_t octets_octets, void* espace, size_t espace_octets, void* flux);

/* The symbol counts of n experts added into `comptes` (device u64[3][4][256]: per matrix j,
 * [0] DELTA, [1 + k] CODES_CTX of scale class k, padding counted): trc_comptes_matrice on the
 * GPU for every matrix of every expert of the batch (lib.rs:393-401). Only blocs[] of the
 * descriptors is read. Asynchronous on `flux`. */
int trc_comptes_gpu(const trc_desc_codage* descs, size_t descs_octets, uint32_t n, const trc_dims_expert* dims,
                    int canonique, uint64_t* comptes, size_t comptes_octets, void* flux);

/* ---------------------------------------------------------------- the expert cache (trc-cache) */

/* The two-tier expert cache of the streaming path (moteur/crates/trc-cache/src/lib.rs:105-301):
 * `emplacements` device slots, `tiedes` host entries of coded parts (0: no host tier), an LRU
 * (politiques.rs:47-160) or Belady (politiques.rs:162-260, it reads the future from the trace it
 * is given: replays only) order per tier. Host code; not thread-safe. */
typedef struct trc_cache trc_cache;

#define TRC_POLITIQUE_LRU 0u
#define TRC_POLITIQUE_BELADY 1u

#define TRC_DECISION_SUCCES 0u        /* the expert is (or will be, in flight) in `emplacement` */
#define TRC_DECISION_DEFAUT_RAM 1u    /* device miss; its coded part is in host entry `tiede` */
#define TRC_DECISION_DEFAUT_DISQUE 2u /* full miss: read it (into host entry `tiede` if >= 0) */

/* Decision (lib.rs:73-82): 16 bytes. */
typedef struct trc_decision {
    uint32_t sorte;       /* TRC_DECISION_* */
    uint32_t emplacement; /* device slot */
    int32_t tiede;        /* host entry, or -1 */
    uint32_t reserve;
} trc_decision;

/* Compteurs (lib.rs:85-99) plus the host tier's evictions: succes_vram + succes_ram +
 * defauts_disque = accesses; bytes are counted only after trc_cache_fixer_tailles. */
typedef struct trc_compteurs_cache {
    uint64_t succes_vram, succes_ram, defauts_disque, octets_disque, octets_copies, evictions, evictions_ram;
} trc_compteurs_cache;

/* A routing trace's dimensions (trace.rs:27-41), or its error: erreur 1 = a malformed line
 * (erreur_ligne), 2 = an expert out of [0, E) (erreur_expert), 3 = empty. */
typedef struct trc_trace_dims {
    uint32_t experts, couches, k, jetons;
    uint32_t erreur, erreur_ligne, erreur_expert, reserve;
} trc_trace_dims;

/* A new cache (Cache::nouveau). Belady needs the trace it will replay: choix[T][L][k] ids
 * (ignored for LRU). `casser` != 0: the policies are not told of hits (the reference's broken
 * policy witness: LRU becomes FIFO). NULL on a usage error. */
trc_cache* trc_cache_nouveau(uint32_t emplacements, uint32_t tiedes, uint32_t politique, const uint16_t* choix,
                             uint32_t jetons, uint16_t couches, uint16_t k, uint32_t casser);
void trc_cache_detruire(trc_cache* cache);
/* Part sizes per (layer, expert): tailles[couche * experts + expert] (Cache::fixer_tailles). */
int trc_cache_fixer_tailles(trc_cache* cache, const uint64_t* tailles, uint16_t couches, uint16_t experts);
/* Serves layer `couche`'s experts at instant t (Cache::demander): pins them, one decision each,
 * in order. TRC_ERR_USAGE when a miss finds no free or evictable slot (the cache is then
 * unusable, as after the reference's panic). */
int trc_cache_demander(trc_cache* cache, uint16_t couche, const uint16_t* experts, uint32_t n, uint64_t t,
                       trc_decision* decisions);
/* The slot's part has landed (Cache::pret): in flight -> present. */
int trc_cache_pret(trc_cache* cache, uint32_t emplacement);
/* The layer's GEMVs are done (Cache::liberer): its experts are unpinned. */
int trc_cache_liberer(trc_cache* cache, uint16_t couche);
void trc_cache_compteurs(const trc_cache* cache, trc_compteurs_cache* sortie);
/* A slot's state: 0 free, 1 in flight, 2 present; niveau 1 (exact) unless free. */
int trc_cache_etat(const trc_cache* cache, uint32_t emplacement, uint32_t* etat, uint32_t* niveau);
/* couche << 16 | expert of a slot's occupant, or -1. */
int64_t trc_cache_occupant(const trc_cache* cache, uint32_t emplacement);
/* The device slot / host entry of an expert, or -1. */
int64_t trc_cache_emplacement_de(const trc_cache* cache, uint16_t couche, uint16_t expert);
int64_t trc_cache_tiede_de(const trc_cache* cache, uint16_t couche, uint16_t expert);
/* The pinned experts (couche << 16 | expert) in pinning order; returns their count. */
uint32_t trc_cache_epingles(const trc_cache* cache, uint32_t* ids, uint32_t capacite);
/* rejouer (lib.rs:272-301): the trace through a new cache, counted in accesses. */
int trc_rejouer(const uint16_t* choix, uint32_t jetons, uint16_t couches, uint16_t k, uint32_t emplacements,
                uint32_t tiedes, uint32_t politique, uint32_t casser, trc_compteurs_cache* sortie);
/* Trace::depuis_texte (trace.rs:43-133): dims (or the error) into *dims; the T * L * k ids into
 * `choix` when capacite (in ids) allows. */
int trc_trace_lire(const char* texte, size_t n, trc_trace_dims* dims, uint16_t* choix, size_t capacite);

/* ---------------------------------------------------------------- the streaming executor (trc-ordo) */

/* MoE layers whose experts' parts live in host memory and come to the GPU on demand
 * (trc-ordo's on-demand step, moteur/crates/trc-ordo/src/lib.rs:1054-1367): a pool of
 * `emplacements` device slots holding parts, managed by the LRU expert cache; per layer call the
 * routed experts are served, each miss copied from the host tier on the executor's copy stream
 * (after the last launch that read its slot), and the fused layer runs on the compute stream
 * once the copies landed. The caller owns every buffer; the executor creates its copy stream,
 * events and a small pinned staging area. Host code; one thread. */
typedef struct trc_flux trc_flux;

typedef struct trc_flux_config {
    uint32_t couches, experts;   /* layers, experts per layer (<= 65,535 each) */
    uint32_t k, jetons_max;      /* routed experts per token (1..8), tokens per call (1..128) */
    trc_dims_expert dims;
    uint32_t emplacements;       /* device part slots, >= k * jetons_max */
    uint32_t n_delta, n_codes;   /* tile lengths of the parts (0: 256) */
    uint32_t reserve;
    uint64_t taille_emplacement; /* bytes per slot: >= every part, a multiple of 256 */
    uint64_t emplacements_carte; /* device: emplacements * taille_emplacement bytes, 256-aligned */
    uint64_t parties_hote;       /* host: u64 [couches][experts], each part's address in host memory
                                    (pinned for the copies to overlap) */
    uint64_t tailles_parties;    /* host: u64 [couches][experts], their sizes */
    uint64_t luts;               /* device: u32 [couches][3][4][4096] */
    uint64_t routeurs;           /* device: f32 [couches][experts][colonnes[0]], or 0 (imposed routing) */
    uint64_t biais_routeurs;     /* device: f32 [couches][experts] */
    uint64_t espace;             /* device workspace, trc_flux_espace_octets bytes, 256-aligned */
    uint64_t flux;               /* the compute stream (cudaStream_t) */
} trc_flux_config;

/* One layer call: distinct experts served, hits, misses, bytes copied, host wait for the router. */
typedef struct trc_flux_stats {
    uint32_t uniques, succes, defauts, reserve;
    uint64_t octets_copies;
    double attente_routeur_s;
} trc_flux_stats;

uint64_t trc_flux_espace_octets(const trc_flux_config* config);
trc_flux* trc_flux_nouveau(const trc_flux_config* config);
void trc_flux_detruire(trc_flux* flux);
/* Layer `couche` on x [jetons][d] (bf16 or f32), residu [jetons][d] f32 updated in place. The
 * routing: experts_imposes / poids_imposes (host [jetons][k]) when given (a routing trace),
 * else the layer's router (the host waits for it). The cache's instant is pas * couches +
 * couche, pas counting calls of the last layer. Asynchronous except for that wait. */
int trc_flux_couche(trc_flux* flux, uint32_t couche, const void* x, uint32_t x_bf16, float* residu, uint32_t jetons,
                    const uint32_t* experts_imposes, const float* poids_imposes, trc_flux_stats* stats);
int trc_flux_compteurs(const trc_flux* flux, trc_compteurs_cache* sortie);
/* The integrity counters u32[4 * k * jetons_max] accumulated over every call (synchronous copy). */
int trc_flux_controle(const trc_flux* flux, uint32_t* sortie, uint32_t n);

/* ---------------------------------------------------------------- the whole decode step (trc-modele) */

/* Row `ligne` of a Q8_0 matrix (34-byte blocks) of `colonnes` columns into y f32[colonnes],
 * exact. Replaces `Noyaux::ligne_q8_0` (trc-noyaux/src/lib.rs:478-486; passe.cuh:623-634). */
int trc_ligne_q8_0(const void* w, size_t w_octets, uint32_t ligne, uint32_t colonnes, float* y, size_t y_octets, void* flux);

/* Index of the largest of n floats into *sortie (u32): ties to the smallest index, a NaN never
 * chosen (all NaN: 0xFFFFFFFF). Replaces `Noyaux::argmax` (lib.rs:488-496; passe.cuh:636-669). */
int trc_argmax(const float* v, size_t v_octets, uint32_t n, uint32_t* sortie, size_t sortie_octets, void* flux);

/* One layer's tensors on the device (the reference's `Couche` of trc-modele/src/lib.rs:400-418):
 * 160 bytes. f32 vectors, Q8_0 matrices, f16 KV caches of `anneau` cases (sliding layers) or of
 * the context; the experts' parts table (u64 addresses and sizes) and the layer's LUTs; `deltas`:
 * the layer's delta bytes decoded ahead (trc_moe_predecoder_deltas) or 0. */
typedef struct trc_modele_couche {
    uint64_t attn_norm, wq, bq, wk, bk, wv, bv, wo, bo, puits, post_norm, wr, br;
    uint64_t cache_k, cache_v;
    uint64_t parties, parties_octets, luts;
    uint32_t anneau, reserve;
    uint64_t deltas;
} trc_modele_couche;

/* The model (`Hyper` + the resident tensors, trc-modele/src/lib.rs:60-83, 342-356): 176 bytes. */
typedef struct trc_modele_config {
    uint32_t couches, d, tetes, tetes_kv, dim_tete, experts, k, vocab, contexte;
    uint32_t brut;             /* 1: the parts are raw (ECHELLES_BRUTES / CODES_BRUTS / BIAIS) */
    uint32_t n_delta, n_codes; /* tile lengths of the parts (0: 256) */
    float eps;
    uint32_t reserve;
    trc_params_rope rope;
    trc_dims_expert dims;
    uint64_t couches_desc;     /* host: trc_modele_couche[couches] */
    uint64_t enchassement;     /* device: Q8_0 [vocab][d] */
    uint64_t norme_sortie;     /* device: f32 [d] */
    uint64_t sortie;           /* device: Q8_0 [vocab][d] */
    uint64_t espace;           /* device workspace, trc_modele_espace_octets bytes, 256-aligned */
    uint64_t espace_octets;
} trc_modele_config;

uint64_t trc_modele_espace_octets(const trc_modele_config* m);
/* Device addresses of the last step's logits (f32[vocab]), greedy token (u32) and the MoE
 * integrity counters (u32[4 k], accumulated; zero them with the workspace). */
int trc_modele_sorties(const trc_modele_config* m, uint64_t* logits, uint64_t* jeton, uint64_t* controle);
/* One token at `position` (Modele::enchasser, debut_couche + the fused layer per layer,
 * sortie; trc-modele/src/lib.rs:476-568), asynchronous on `flux`; sortie = 0 skips the
 * unembedding (a context token). */
int trc_modele_pas(const trc_modele_config* m, uint32_t jeton, uint32_t position, uint32_t sortie, void* flux);

/* The step in phases, for a caller that puts an exchange between them (the expert-parallel
 * model: the MoE input of every rank's token gathered, the layer run on each rank's expert
 * share, the sums scattered back). trc_modele_pas = debut, then per layer attention + moe, then
 * fin, launch for launch.
 *   debut:     x <- row `jeton` of the embedding (Modele::enchasser, lib.rs:476-480);
 *   attention: layer `couche`'s attention side at `position`, x += o, then h2 <- RMSNorm(x), the
 *              MoE's input (Modele::debut_couche, lib.rs:482-531);
 *   moe:       router, top-k, the fused layer on h2, x += the weighted experts (fin_couche);
 *   fin:       RMSNorm, unembedding, greedy token (Modele::sortie, lib.rs:555-568).
 * trc_modele_etat gives the device addresses of x and h2 (f32[d] each) in the workspace. */
int trc_modele_debut(const trc_modele_config* m, uint32_t jeton, void* flux);
int trc_modele_attention(const trc_modele_config* m, uint32_t couche, uint32_t position, void* flux);
int trc_modele_moe(const trc_modele_config* m, uint32_t couche, void* flux);
int trc_modele_fin(const trc_modele_config* m, void* flux);
int trc_modele_etat(const trc_modele_config* m, uint64_t* x, uint64_t* h2);

/* trc_modele_attention for n sequences of one model at the same position (each its own KV caches
 * and workspace, the same weights: checked), the q / k / v and output Q8_0 GEMVs launched once
 * for the n tokens (each weight row read once); every sequence gets trc_modele_attention's bits.
 * `espace`: trc_modele_lot_espace_octets(m, n) bytes, 256-aligned. */
uint64_t trc_modele_lot_espace_octets(const trc_modele_config* m, uint32_t n);
int trc_modele_attention_lot(const trc_modele_config* const* sequences, uint32_t n, uint32_t couche, uint32_t position,
                             void* espace, size_t espace_octets, void* flux);

/* Seeded synthetic tensors on the GPU (inputs of tests and benches; no counterpart): R x C
 * MXFP4 as 17-byte blocks + f32 biases (row sigma 0.02 LogNormal(0, 0.3), E8M0 floor(log2 max)
 * - 2, E2M1 to nearest, biases N(0, 0.01) rounded to bf16); R x C Q8_0 of N(0, 0.02); n f32
 * moyenne + ecart N(0, 1). `matrice` / `flux_id` name the stream of draws. */
int trc_synth_mxfp4_gpu(uint8_t* blocs, float* biais, uint32_t lignes, uint32_t colonnes, uint64_t graine,
                        uint64_t matrice, void* flux);
int trc_synth_q8_0_gpu(uint8_t* w, uint32_t lignes, uint32_t colonnes, uint64_t graine, uint64_t matrice, void* flux);
int trc_synth_f32_gpu(float* y, uint64_t n, uint64_t graine, uint64_t flux_id, float moyenne, float ecart, void* flux);
/* Raw parts of n experts from their blocks (descs: blocs, biais, sortie, expert), `taille`
 * bytes each: `entete` (the header and stream table trc_coder_partie_brute writes, with any
 * expert number) then the streams at its offsets, zeros elsewhere. */
int trc_parties_brutes_gpu(const trc_desc_codage* descs, uint32_t n, const trc_dims_expert* dims, const uint8_t* entete,
                           uint32_t entete_octets, uint64_t taille, void* flux);

/* ---------------------------------------------------------------- new: the fused MoE layer */

/* One MoE layer of one token, fused: routed experts' DELTA -> scales, CODES_CTX decoded in
 * registers and multiplied at once (gate, up), SwiGLU, then down, then the weighted combine
 * into the residual. The decoded nibbles and scales never go to the slot layout in HBM. No
 * reference counterpart (the reference decodes into slots, then runs gemv, swiglu_oai and
 * combiner: trc-modele/src/lib.rs:533-553). Bit for bit the same result as trc_decoder_lot +
 * trc_gemv + trc_swiglu_oai + trc_combiner on the same weights, and as the raw path (`brut`)
 * on the raw parts of the same experts. */
typedef struct trc_moe_couche {
    const uint64_t* parties;        /* device u64[experts]: each expert's level-0 part (16-aligned) */
    const uint64_t* parties_octets; /* device u64[experts]: their sizes */
    uint32_t experts;               /* experts of the layer */
    uint32_t k;                     /* active experts per token (<= 8) */
    const uint32_t* luts;           /* device: the layer's u32[3][4][4096] (unused when brut) */
    trc_dims_expert dims;           /* hidden d = colonnes[0] = colonnes[1] = lignes[2];
                                       ffn width f = lignes[0] = lignes[1] = colonnes[2] */
    const uint32_t* indices;        /* device u32[k]: the chosen experts (router output) */
    const float* poids;             /* device f32[k]: their weights */
    const void* x;                  /* device activation [d], bf16 (x_bf16 = 1) or f32 */
    uint32_t x_bf16;
    uint32_t brut;                  /* 1: raw parts (ECHELLES_BRUTES / CODES_BRUTS / BIAIS) */
    float* residu;                  /* device f32[d]: updated in place */
    uint32_t* controle;             /* device u32[4*k]: counters per active expert, zeroed by caller */
    uint32_t n_delta, n_codes;      /* macro-steps per tile the parts were encoded with (0: 256, what
                                       trc-codeur writes); they only size the grids */
    /* Token batch and expert parallelism (all zero: one token, every expert held here). */
    uint32_t jetons;                /* tokens (0 = 1): x is [jetons][d], residu [jetons][d], indices /
                                       poids / controle hold jetons * k activations, token-major */
    uint32_t expert_debut;          /* experts held by this call: [expert_debut, expert_fin); the */
    uint32_t expert_fin;            /* others are skipped, no error (expert_fin = 0: all are held) */
    uint32_t partiel;               /* 1: residu[b] = this call's weighted sum over its held
                                       activations (0 when none), for a sum across GPUs; 0: residu += */
    const struct trc_echange_pairs* echange; /* host pointer or NULL: the combine's sum across
                                       GPUs done by the combine kernel itself over peer memory */
    const uint8_t* deltas;          /* device or NULL: the delta bytes of every expert of the layer,
                                       decoded ahead by trc_moe_predecoder_deltas (then the layer
                                       skips its DELTA phase; same results); ignored when brut */
} trc_moe_couche;

/* The combine's exchange between the GPUs of an expert-parallel layer, in the combine kernel:
 * each rank's combine writes its share of every token's weighted sum into its slot of every
 * rank's exchange buffer (peer stores over NVLink), raises a flag there, waits for every rank's
 * flag on its own buffer (bounded: a wait that gives up counts in controle[3] of activation 0
 * and leaves the residual unchanged), then adds the shares in rank order: every rank ends with
 * the same residual, bit for bit. The buffers are one per rank, of trc_echange_octets bytes,
 * mapped in every rank's address space (e.g. symmetric memory), zeroed once before the first
 * call; every rank calls the layer the same number of times, with the same tokens. */
typedef struct trc_echange_pairs {
    uint64_t tampons[8];  /* device addresses, in this process, of the exchange buffers of ranks
                             0 .. monde-1 (tampons[rang] is this rank's own) */
    uint32_t rang;        /* this rank */
    uint32_t monde;       /* ranks (2 .. 8) */
} trc_echange_pairs;

/* Bytes of one rank's exchange buffer for these dimensions, tokens per call and ranks. */
uint64_t trc_echange_octets(const trc_dims_expert* dims, uint32_t jetons, uint32_t monde);

/* Workspace bytes the fused layer needs for these dimensions and k activations (tokens times
 * routed experts per token; device memory the caller allocates once and reuses; contents need no
 * initialisation). */
uint64_t trc_moe_espace_octets(const trc_dims_expert* dims, uint32_t k);

/* Workspace bytes with which the fused layer takes its overlapped schedule (k <= 32 activations;
 * beyond, trc_moe_espace_octets): every CODES_CTX tile of the three matrices decoded in one
 * launch, the decoded code words through the workspace (16 bytes per MXFP4 block and activation:
 * 49.8 MB more for gpt-oss at k = 4, 53,199,360 bytes in all), then the GEMVs on them. Given at
 * least this, the layer takes that schedule; given less (but at least trc_moe_espace_octets),
 * the sequential one. Both give the same bits. */
uint64_t trc_moe_espace_recouvrant_octets(const trc_dims_expert* dims, uint32_t k);

/* Runs the fused layer. `espace` (256-aligned) >= trc_moe_espace_octets (see
 * trc_moe_espace_recouvrant_octets for the faster schedule). Compressed parts need
 * CODES_CTX tiles whose N is a multiple of 32 (trc-codeur writes 256); other N are counted as
 * format errors (decode them with trc_decoder_expert instead). */
int trc_moe_couche_fusionnee(const trc_moe_couche* couche, void* espace, size_t espace_octets, void* flux);

/* Workspace bytes of trc_moe_couche_par_flux for these dimensions, experts per layer and
 * activations (tokens x k): a decoded slot per distinct routed expert (at most
 * min(activations, experts); 13,254,144 bytes each for gpt-oss) and per-activation vectors. */
uint64_t trc_moe_par_flux_espace_octets(const trc_dims_expert* dims, uint32_t experts, uint32_t activations);

/* The layer over a batch of positions "par flux" (the reference's prefill by stream,
 * trc-modele/src/lib.rs:607-717, trc-ordo/src/lib.rs:782-981): each distinct routed expert is
 * decoded once for the whole batch into a slot of the workspace, then applied to every position
 * routed to it with the token-by-token arithmetic, so the residuals are bit-identical to
 * trc_moe_couche_fusionnee's on the same descriptor. Compressed parts, or raw parts (brut: each
 * distinct expert's streams copied into its slot, the same bits); no exchange;
 * an expert share (expert_debut / expert_fin: the other experts' activations left out) and
 * partiel (each position's share of the sum written alone) are those of the fused layer. The
 * controle of an activation receives its expert's decode counters. Up to 4,096 positions per
 * call (the fused layer: 128). */
int trc_moe_couche_par_flux(const trc_moe_couche* couche, void* espace, size_t espace_octets, void* flux);

/* New: workspace bytes of trc_moe_couche_par_flux_mma (trc_moe_par_flux_espace_octets plus the
 * GEMMs' quantized activations). */
uint64_t trc_moe_par_flux_mma_espace_octets(const trc_dims_expert* dims, uint32_t experts, uint32_t activations,
                                            uint32_t seuil);

/* New: the layer par flux with every expert that receives at least `seuil` activations of the
 * batch (16 and up is where it pays) multiplied on the tensor cores (trc_gemm_mxfp4's
 * tcgen05 block-scaled GEMM over the expert's decoded slot, x and h quantized to MXFP8, the rows
 * gathered and scattered through the expert's activation list); the other experts as
 * trc_moe_couche_par_flux. Not bit-identical to it (about 3 % of the layer's output, the
 * quantization). The call waits on `flux` once, for the routing (read
 * back to size the GEMMs): it cannot be captured in a CUDA graph. Raw parts as in
 * trc_moe_couche_par_flux. *erreur (device u32, zeroed by
 * the caller) is set to 1 when a bounded wait of the GEMM kernel gave up. */
int trc_moe_couche_par_flux_mma(const trc_moe_couche* couche, uint32_t seuil, void* espace, size_t espace_octets,
                                uint32_t* erreur, void* flux);

/* New: bytes of a layer's delta bytes decoded ahead (trc_moe_predecoder_deltas): one byte per
 * 32-block of each matrix and expert, 256-aligned per matrix (3 x 259,200 x 128 = 99.5 MB for a
 * gpt-oss-120b layer of 128 experts, against about 76.8 MB of DELTA streams). */
uint64_t trc_moe_deltas_octets(const trc_dims_expert* dims, uint32_t experts);

/* New: decodes the DELTA stream of every matrix of every expert of a layer (the first half of
 * trc-codec's decoder_matrice_v10, lib.rs:190-212, as the fused layer's DELTA phase does it)
 * into `deltas` (trc_moe_deltas_octets bytes): the weights' scale offsets, which need no
 * activation, decoded once at load instead of at every step. Only parties, parties_octets,
 * experts, luts, dims and n_delta of `couche` are read; controle: device u32[4 x experts],
 * zeroed by the caller, the counters of each expert's DELTA streams. Passing the result as
 * couche->deltas removes the DELTA phase from trc_moe_couche_fusionnee. Async on the stream. */
int trc_moe_predecoder_deltas(const trc_moe_couche* couche, uint8_t* deltas, uint64_t deltas_octets,
                              uint32_t* controle, void* flux);

/* ---------------------------------------------------------------- the tensor-core expert GEMM */

/* New (the reference multiplies one token at a time, gemv_mxfp4, gemv.cuh:140-161; its prefill
 * par flux applies the per-token GEMV to every position routed to an expert,
 * trc-modele/src/lib.rs:607-717): for an expert receiving many tokens at once,
 * y[t][r] = sum_c W[r][c] x[t][c] + biais[r] on the tensor cores (tcgen05.mma,
 * kind::mxf8f6f4.block_scale): W the matrix in the slot / raw-part layout (codes: 16 bytes per
 * 32-block, row-major, 16-aligned; echelles: one E8M0 byte per block, 16-aligned; biais f32[lignes] or NULL),
 * x [n][colonnes] f32 or bf16, quantized on the GPU to MXFP8 (E4M3 elements, one E8M0 scale per 32:
 * 2^(floor(log2 max|x|) - 8)); f32 accumulation. n = 1 to 256 tokens (the MMA's N, padded to 16);
 * espace: trc_gemm_mxfp4_espace_octets bytes, 256-aligned (the quantized x). Not bit-identical
 * to the GEMV (x is quantized): within the tolerance the tests state. *erreur (device u32,
 * zeroed by the caller) is set to 1 when a bounded wait of the kernel gave up. */
int trc_gemm_mxfp4(const uint8_t* codes, const uint8_t* echelles, const float* biais, uint32_t lignes, uint32_t colonnes,
                   const void* x, uint32_t x_bf16, uint32_t n, float* y, void* espace, size_t espace_octets,
                   uint32_t* erreur, void* flux);
uint64_t trc_gemm_mxfp4_espace_octets(uint32_t colonnes, uint32_t n);

/* New: one matrix of a batch of trc_gemm_mxfp4 calls, 56 bytes (device addresses). Each matrix
 * must meet trc_gemm_mxfp4's rules (codes and scales 16-aligned, colonnes a multiple of 32, 1 to
 * 256 tokens); trc_gemm_mxfp4_lot checks them. Codes 32-aligned with colonnes a multiple of 64
 * let the weight tiles come by TMA (otherwise 8-byte copies). */
typedef struct trc_desc_gemm {
    uint64_t codes, echelles, biais, x, y;
    uint32_t lignes, colonnes, n, x_bf16;
} trc_desc_gemm;

/* New: nb tensor-core GEMMs, two launches per group of up to 48 matrices (every x quantized,
 * then every matrix's row tiles): descs HOST trc_desc_gemm[nb] (copied into the launches'
 * parameters with each matrix's TMA tensor maps; the caller may reuse the array on return), rows
 * / columns / tokens of each at most lignes_max / colonnes_max / n_max; espace
 * trc_gemm_mxfp4_lot_espace_octets bytes, 256-aligned. For the experts of a layer that receive
 * many tokens (an expert-parallel share at batch 64). */
int trc_gemm_mxfp4_lot(const trc_desc_gemm* descs, uint32_t nb, uint32_t lignes_max, uint32_t colonnes_max,
                       uint32_t n_max, void* espace, size_t espace_octets, uint32_t* erreur, void* flux);
uint64_t trc_gemm_mxfp4_lot_espace_octets(uint32_t colonnes_max, uint32_t n_max, uint32_t nb);

/* ---------------------------------------------------------------- expert parallelism over NCCL */

/* New (the reference is single-GPU; its combine is `combiner`, passe.cuh:611-622, driven by
 * trc-modele/src/lib.rs:533-553): one rank's step of the expert-parallel layer, for a host with
 * one process per GPU and an NCCL communicator `comm` (ncclComm_t) over them. The rank runs
 * trc_moe_couche_fusionnee on the experts it holds (couche->expert_debut / expert_fin; its
 * parts only need to be present for those) with the partial combine (rank 0 adds its share's
 * weighted sum into the residual, the other ranks write their share's sum alone), then one NCCL
 * SUM all-reduce of the [jetons][d] f32 residual on `flux`: every rank ends with residual + the
 * weighted sum over all routed experts (the reference's terms, summed in another order across
 * GPUs). Every rank calls it with the same tokens and routing (a replicated router). partiel and
 * echange must be 0 / NULL (the call sets the first). NCCL is resolved at run time
 * (libnccl.so.2, the host's copy when one is loaded); NCCL errors return TRC_ERR_CUDA with the
 * text in trc_derniere_erreur. */
int trc_moe_couche_ep(const trc_moe_couche* couche, void* espace, size_t espace_octets, void* comm, void* flux);

/* New: the communicator for a host with no NCCL binding of its own. trc_nccl_id writes a unique
 * id (128 bytes) on one rank; after the host has sent it to every rank, each calls
 * trc_nccl_init with its rank (blocks until all ranks have joined) and later trc_nccl_fin. */
int trc_nccl_id(uint8_t* id, size_t id_octets);
int trc_nccl_init(void** comm, uint32_t monde, const uint8_t* id, uint32_t rang);
int trc_nccl_fin(void* comm);

/* trc_moe_couche_fusionnee, recording evenements[0..5] (cudaEvent_t, each may be NULL) on the
 * stream: before the DELTA phase, after it, after gate/up, after SwiGLU, after down, after the
 * combine (raw parts: no DELTA phase, [1] is recorded with [0]). For timing each phase with CUDA
 * events on the launching stream; the launches are those of trc_moe_couche_fusionnee. */
int trc_moe_couche_chrono(const trc_moe_couche* couche, void* espace, size_t espace_octets, void* flux,
                          void* const* evenements);

/* No counterpart in the reference. trc_moe_couche_fusionnee without a workspace argument, for
 * callers that cannot allocate device memory where they run the layer (an FFI caller holding only
 * the buffers it was given, a serving loop whose device memory is fixed up front). The workspace
 * is a fixed 8 MiB (8,388,608-byte) area of this library's device memory, one per device: a layer
 * whose trc_moe_espace_octets exceeds it is refused with TRC_ERR_USAGE before any launch. Nothing
 * is allocated. The first call on each device looks up the area's address there, so make it
 * before any stream capture; that address is kept for the process's life, so do not call this on
 * a device reset (cudaDeviceReset) since its first call there. All calls on a device share the area: calls that may overlap in
 * time (different streams, different threads) race on it; calls on one stream are safe. Nothing
 * in the area needs zeroing. Results and launches are those of trc_moe_couche_fusionnee. */
int trc_moe_couche_sans_alloc(const trc_moe_couche* couche, void* flux);

/* Router of the layer for `jetons` tokens (1 to 4,096; x [jetons][colonnes], bf16 or f32): logits = Wr x + br
 * (f32 weights [experts][colonnes]), then top-k and f64 softmax as trc_routeur_topk, token by
 * token: logits f32[jetons][experts], indices u32[jetons][k], poids f32[jetons][k]. Two launches
 * whatever the number of tokens. */
int trc_routeur(const float* wr, const float* br, const void* x, uint32_t x_bf16, uint32_t experts,
                uint32_t colonnes, uint32_t k, uint32_t jetons, float* logits, uint32_t* indices, float* poids,
                void* flux);

/* ---------------------------------------------------------------- the quality judge (trc-juge) */

/* u16 words of one `.kld` logit entry of n_vocab logits: 2 ceil(n_vocab / 2) + 4
 * (`kld::mots_par_entree`, trc-juge/src/kld.rs:27-29). */
uint64_t trc_juge_mots_par_entree(uint32_t n_vocab);

/* Codes n_positions rows of logits (f32, or f64 when f64 = 1; row-major [n_positions][n_vocab])
 * into consecutive `.kld` entries (sortie: n_positions x trc_juge_mots_par_entree words, the
 * file's layout), the rule of `kld::coder_entree` (kld.rs:148-186) with every intermediate in
 * f64. One launch. */
int trc_juge_coder(const void* logits, uint32_t f64, size_t logits_octets, uint32_t n_positions, uint32_t n_vocab,
                   uint16_t* sortie, size_t sortie_octets, void* flux);

/* One judged position (`stats::Position`, trc-juge/src/stats.rs:24-33): 48 bytes. */
typedef struct {
    double kl;               /* KL(P || Q) over log p_i > -16 */
    double nll_q, nll_p;     /* NLL of the next token under Q and under P */
    double dp;               /* q(next) - p(next) */
    uint32_t premier_p, premier_q;  /* argmax, ties to the first index */
    uint32_t meme_premier;   /* premier_p == premier_q */
    uint32_t suivant_valide; /* 0: the next token was >= n_vocab (NLLs and dp are NaN) */
} trc_juge_position;

/* KL, first choice and NLLs of n_positions positions: P = coded entries (n_positions x nv words);
 * Q per `mode`: 0 = coded entries, taken as log-probabilities without renormalisation
 * (`stats::position_decodee`, stats.rs:33-39); 1 = raw f32 logits [n_positions][n_vocab]; 2 = raw
 * f64 logits (both renormalised by their log-sum-exp: `stats::position`, stats.rs:36-85).
 * suivants u32[n_positions] = the next token of each position. One launch. */
int trc_juge_positions(const uint16_t* p, size_t p_octets, const void* q, size_t q_octets, uint32_t mode,
                       const uint32_t* suivants, size_t suivants_octets, uint32_t n_positions, uint32_t n_vocab,
                       trc_juge_position* sortie, size_t sortie_octets, void* flux);

#ifdef __cplusplus
}
#endif

#endif /* TRONCONS_B200_H */
