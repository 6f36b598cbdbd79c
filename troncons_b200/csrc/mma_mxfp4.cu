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
// are copied as they are into the unpacked shared-memory form of 4-bit operands (16 elements in
// 8 bytes, then 8 bytes of padding, per 16 bytes).
//
// Shared memory, K-major without swizzle: 8-row x 16-byte core matrices, the next core matrix
// along K 128 bytes further (LBO), the next 8 rows 1,024 bytes further (SBO), one chunk of 128 K
// (four MMAs) at a time. Scale factors in tensor memory, the layout of tcgen05.cp's 32x128b
// copies replicated to the four lane quadrants: lane (m mod 32), column m / 32 + base, byte =
// the 32-block within the chunk (the instruction descriptor's and the address's scale-factor id).
//
// One CTA of 4 warps per 128-row tile: the warps stage chunks (cp.async of the weight halves and
// the quantized activations, three or four stages, two chunks ahead) and write their scale factors
// to tensor memory, thread 0 issues each chunk's MMAs and commits them to the stage's mbarrier,
// which every thread waits on (bounded) before that stage is refilled; the epilogue reads the accumulator (tcgen05.ld), adds the bias and stores Y. Every wait
// is bounded: a wait that gives up sets the caller's error word, waits again (bounded) for the
// MMAs in flight, frees the tensor memory and returns.
#include <cstdint>

#include "commun.cuh"
#include "noyaux.h"

namespace tb {

constexpr uint32_t MMA_M = 128;        // rows per CTA (one MMA's M); chunks of 128 K (four MMAs)
constexpr uint32_t MMA_FILS = 128;     // four warps: one per tensor-memory lane quadrant

// Stages of 128 K: E = 4 where shared memory holds them, else 3. The chunk loaded at step ch is
// ch + E - 2, into the stage chunk ch - 2 used: its MMAs, issued two steps before, are done.
constexpr uint32_t MMA_ETAGES_MAX = 4;

__host__ __device__ __forceinline__ uint32_t mma_n_pad(uint32_t N) { return (N + 15u) & ~15u; }
// Tensor-memory columns: the accumulator (Npad), then per stage SFA (4) and SFB (8).
__host__ __device__ __forceinline__ uint32_t mma_tmem_colonnes(uint32_t N, uint32_t E) {
    const uint32_t besoin = mma_n_pad(N) + 12u * E;
    uint32_t c = 32u;
    while (c < besoin) c <<= 1;
    return c;
}
// Shared bytes of one stage: A tile (128 rows x 128 bytes) and B tile (Npad rows x 128 bytes).
__host__ __device__ __forceinline__ uint32_t mma_etage(uint32_t N) { return MMA_M * 128u + mma_n_pad(N) * 128u; }
// Scale bytes of the CTA's 128 rows and of the tokens (staged once), 16-aligned.
__host__ __device__ __forceinline__ uint32_t mma_echelles(uint32_t N, uint32_t C) {
    return ((MMA_M + mma_n_pad(N)) * (C / 32u) + 15u) & ~15u;
}
// All stages, the staged scales, the mbarriers and the tensor-memory base.
__host__ __device__ __forceinline__ uint32_t mma_smem(uint32_t N, uint32_t C, uint32_t E) {
    return E * mma_etage(N) + mma_echelles(N, C) + 64u;
}
// Four stages where two CTAs still fit on an SM (their chunks interleave), else three.
__host__ __device__ __forceinline__ uint32_t mma_etages(uint32_t N, uint32_t C) {
    return mma_smem(N, C, 4u) <= 112u * 1024u ? 4u : 3u;
}

// Offset in a K-major no-swizzle tile of row r and byte k (0..127) of the chunk.
__device__ __forceinline__ uint32_t mma_off(uint32_t r, uint32_t k) {
    return (r >> 3) * 1024u + (k >> 4) * 128u + (r & 7u) * 16u + (k & 15u);
}

__device__ __forceinline__ uint64_t mma_desc(uint32_t adresse) {
    uint64_t d = 0;
    d |= uint64_t((adresse >> 4) & 0x3FFFu);
    d |= uint64_t(128u >> 4) << 16;   // leading byte offset: the next core matrix along K
    d |= uint64_t(1024u >> 4) << 32;  // stride byte offset: the next 8 rows
    d |= uint64_t(1) << 46;           // descriptor version of sm_100
    return d;                         // base offset 0, no swizzle
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

// The weight halves of rows r0 .. r0 + 127, 32-blocks kb0 .. kb0 + nkb - 1, into the A tile.
__device__ __forceinline__ void charger_a(uint8_t* ta, const uint8_t* codes, uint32_t R, uint32_t B, uint32_t r0,
                                          uint32_t kb0, uint32_t nkb) {
    for (uint32_t t = threadIdx.x; t < MMA_M * 4u * 2u; t += MMA_FILS) {
        const uint32_t r = t >> 3, kb = (t >> 1) & 3u, h = t & 1u;
        if (kb >= nkb || r0 + r >= R) continue;
        const uint8_t* src = codes + (uint64_t(r0 + r) * B + kb0 + kb) * 16u + 8u * h;
        cp_async8(ta + mma_off(r, 32u * kb + 16u * h), src);
    }
}

// The quantized activations of the chunk (32 bytes per token and block) into the B tile.
__device__ __forceinline__ void charger_b(uint8_t* tb_, const uint8_t* xq, uint32_t C, uint32_t N, uint32_t kb0,
                                          uint32_t nkb) {
    for (uint32_t t = threadIdx.x; t < N * 4u * 2u; t += MMA_FILS) {
        const uint32_t n = t >> 3, kb = (t >> 1) & 3u, h = t & 1u;
        if (kb >= nkb) continue;
        cp_async16(tb_ + mma_off(n, 32u * kb + 16u * h), xq + uint64_t(n) * C + 32u * (kb0 + kb) + 16u * h, 16u);
    }
}

// Scale bytes of row (or token) m of the staged scales for blocks kb0 .. kb0 + 3 (0 beyond nkb or
// past `lignes`).
__device__ __forceinline__ uint32_t quatre_echelles(const uint8_t* ech_s, uint32_t m, uint32_t lignes, uint32_t B,
                                                    uint32_t kb0, uint32_t nkb) {
    if (m >= lignes) return 0u;
    uint32_t v = 0;
    for (uint32_t k = 0; k < nkb; ++k) v |= uint32_t(ech_s[m * B + kb0 + k]) << (8u * k);
    return v;
}

// n bytes (n a multiple of 16, both addresses 16-aligned) into shared memory by 16-byte cp.async.
__device__ __forceinline__ void copier_async(uint8_t* dst, const uint8_t* src, uint32_t n) {
    for (uint32_t t = threadIdx.x; t < n / 16u; t += blockDim.x) cp_async16(dst + 16u * t, src + 16u * t, 16u);
}

struct ArgsMma {
    const uint8_t* codes;  // W: 16 bytes per 32-block, row-major
    const uint8_t* ech;    // W: E8M0 per block
    const float* biais;    // R f32, or null
    const uint8_t* xq;     // X quantized: [N][C] E4M3 in the blocks' MMA order
    const uint8_t* xs;     // X scales: [N][C / 32] E8M0
    float* y;              // [N][R]
    uint32_t R, C, N;
    uint32_t* erreur;      // set to 1 when a bounded wait gave up
};

// Matrix blockIdx.y of a batch: its descriptor (device) and its slice of the workspace.
__device__ __forceinline__ ArgsMma args_du_lot(const DescGemm* __restrict__ lot, uint8_t* espace, uint64_t tranche,
                                               uint32_t* erreur) {
    const DescGemm d = lot[blockIdx.y];
    uint8_t* xq = espace + tranche * blockIdx.y;
    return ArgsMma{reinterpret_cast<const uint8_t*>(d.codes), reinterpret_cast<const uint8_t*>(d.echelles),
                   reinterpret_cast<const float*>(d.biais), xq, xq + uint64_t(mma_n_pad(d.n)) * d.colonnes,
                   reinterpret_cast<float*>(d.y), d.lignes, d.colonnes, d.n, erreur};
}

// One launch: `a` (lot == nullptr), or matrix blockIdx.y of a batch (its rows past its own R
// leave the CTA idle).
__global__ void __launch_bounds__(MMA_FILS, 2) k_gemm_mxfp4(ArgsMma a0, const DescGemm* lot, uint8_t* espace_lot,
                                                            uint64_t tranche, uint32_t E) {
    extern __shared__ __align__(1024) uint8_t dyn[];
    const ArgsMma a = lot != nullptr ? args_du_lot(lot, espace_lot, tranche, a0.erreur) : a0;
    if (blockIdx.x * MMA_M >= a.R || a.N == 0) return;
    const uint32_t Np = mma_n_pad(a.N), etage = mma_etage(a.N);
    uint8_t* ech_a = dyn + E * etage;              // the CTA's rows' scales [128][B]
    uint8_t* ech_b = ech_a + MMA_M * (a.C / 32u);           // the tokens' scales [N][B]
    uint64_t* mb = reinterpret_cast<uint64_t*>(dyn + E * etage + mma_echelles(a.N, a.C));  // per stage
    uint32_t* tmem_base_s = reinterpret_cast<uint32_t*>(mb + E);
    const uint32_t warp = threadIdx.x >> 5, voie = threadIdx.x & 31u;
    const uint32_t r0 = blockIdx.x * MMA_M, B = a.C / 32u;
    const uint32_t ncol = mma_tmem_colonnes(a.N, E);
    const uint32_t col_acc = 0;
    auto col_sfa = [Np](uint32_t e) { return Np + 12u * e; };
    auto col_sfb = [Np](uint32_t e) { return Np + 12u * e + 4u; };

    // Padding bytes (and rows past R or N) stay zero; only the data halves are ever written.
    for (uint32_t i = threadIdx.x; i < E * etage / 16u; i += MMA_FILS)
        reinterpret_cast<uint4*>(dyn)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        for (uint32_t e = 0; e < E; ++e) mbar_init(mb + e, 1u);
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
    attendre_amont();
    liberer_aval();

    const uint32_t nchunks = (B + 3u) / 4u;
    const uint32_t quadrant = (warp & 3u) * 32u;
    // The scales, once: the CTA's rows (contiguous, 16-aligned: r0 B is a multiple of 16) and
    // the tokens'; past R, a partial last tile reads rows of zeros (they are never multiplied).
    {
        const uint32_t lignes = min(MMA_M, a.R - r0);
        copier_async(ech_a, a.ech + uint64_t(r0) * B, (lignes * B) & ~15u);
        for (uint32_t i = ((lignes * B) & ~15u) + threadIdx.x; i < lignes * B; i += MMA_FILS)
            ech_a[i] = a.ech[uint64_t(r0) * B + i];
        copier_async(ech_b, a.xs, (a.N * B) & ~15u);
        for (uint32_t i = ((a.N * B) & ~15u) + threadIdx.x; i < a.N * B; i += MMA_FILS) ech_b[i] = a.xs[i];
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
    }
    // Chunk ch into stage ch % E: the tiles by cp.async (one commit group), the scale
    // factors into the stage's tensor-memory columns.
    auto charger = [&](uint32_t ch) {
        if (ch < nchunks) {
            const uint32_t e = ch % E, kb0 = 4u * ch, nkb = min(4u, B - kb0);
            uint8_t* ta = dyn + e * etage;
            charger_a(ta, a.codes, a.R, B, r0, kb0, nkb);
            charger_b(ta + MMA_M * 128u, a.xq, a.C, a.N, kb0, nkb);
            uint32_t v[4];
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) v[c] = quatre_echelles(ech_a, voie + 32u * c, a.R - r0, B, kb0, nkb);
            tmem_st4(tmem + (quadrant << 16) + col_sfa(e), v[0], v[1], v[2], v[3]);
#pragma unroll
            for (uint32_t c = 0; c < 4; ++c) v[c] = quatre_echelles(ech_b, voie + 32u * c, a.N, B, kb0, nkb);
            tmem_st4(tmem + (quadrant << 16) + col_sfb(e), v[0], v[1], v[2], v[3]);
            if (Np > 128u) {  // tokens 128 .. 255: four more columns
#pragma unroll
                for (uint32_t c = 0; c < 4; ++c) v[c] = quatre_echelles(ech_b, 128u + voie + 32u * c, a.N, B, kb0, nkb);
                tmem_st4(tmem + (quadrant << 16) + col_sfb(e) + 4u, v[0], v[1], v[2], v[3]);
            }
        }
        cp_async_commit();  // an empty group past the last chunk keeps the group count uniform
    };
    // Parity of the k-th completion (k = ch / E) of stage ch % E's mbarrier.
    auto parite = [E](uint32_t ch) { return (ch / E) & 1u; };
    const uint32_t D = E - 2u;  // chunks loaded ahead
    bool ok = true;
    for (uint32_t ch = 0; ch < D; ++ch) charger(ch);
    for (uint32_t ch = 0; ch < nchunks && ok; ++ch) {
        // Chunk ch + D goes into the stage chunk ch - 2 used: its MMAs first.
        if (ch >= 2u) ok = mbar_attendre(mb + (ch - 2u) % E, parite(ch - 2u));
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        charger(ch + D);
        if (D == 2u)  // this thread's copies of chunk ch have landed (groups ch + 1 .. ch + D may not)
            cp_async_wait<2>();
        else
            cp_async_wait<1>();
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
        __syncthreads();
        if (threadIdx.x == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
            const uint32_t e = ch % E, nkb = min(4u, B - 4u * ch);
            const uint32_t ta = adresse_partagee(dyn + e * etage), tbs = ta + MMA_M * 128u;
            for (uint32_t kb = 0; kb < nkb; ++kb) {
                const uint64_t da = mma_desc(ta + 256u * kb);
                const uint64_t db = mma_desc(tbs + 256u * kb);
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
                             adresse_partagee(mb + e))
                         : "memory");
        }
    }
    // The last chunk's MMAs (the accumulator's last writes: MMAs complete in order).
    if (ok) ok = mbar_attendre(mb + (nchunks - 1u) % E, parite(nchunks - 1u));
    cp_async_wait<0>();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
    if (!ok) {
        if (threadIdx.x == 0) atomicExch(a.erreur, 1u);
        // A second bounded wait for the MMAs in flight (the last committed chunk's stage).
        for (uint32_t e = 0; e < E; ++e) mbar_attendre(mb + e, 0u), mbar_attendre(mb + e, 1u);
    } else {
        // Epilogue: warp q reads rows r0 + 32 q + lane, 8 tokens at a time.
        const uint32_t r = r0 + quadrant + voie;
        const float bias = (a.biais != nullptr && r < a.R) ? a.biais[r] : 0.0f;
        for (uint32_t n0 = 0; n0 < Np; n0 += 8u) {
            uint32_t v[8];
            tmem_ld8(tmem + (quadrant << 16) + col_acc + n0, v);
            asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
            if (r < a.R)
                for (uint32_t j = 0; j < 8u; ++j)
                    if (n0 + j < a.N) a.y[uint64_t(n0 + j) * a.R + r] = __uint_as_float(v[j]) + bias;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(ncol) : "memory");
    }
}

// X (f32 or bf16, [N][C]) into MXFP8: per token and 32-block, E = floor(log2 max|x|) - 8 (the
// largest E4M3 exponent), scale byte E + 127 (E = -127 for an all-zero block), elements
// x / 2^E rounded to E4M3 (nearest even, saturating at 448), written in the block's MMA order
// (k' = 2i <- element i, k' = 2i + 1 <- element 16 + i). One warp per (token, block).
__global__ void __launch_bounds__(256) k_quantifier_mxfp8(const void* x, uint32_t bf16, uint32_t C, uint32_t N,
                                                          uint8_t* xq, uint8_t* xs, const DescGemm* lot, uint64_t tranche) {
    attendre_amont();
    liberer_aval();
    if (lot != nullptr) {  // matrix blockIdx.y of a batch
        const DescGemm d = lot[blockIdx.y];
        x = reinterpret_cast<const void*>(d.x);
        bf16 = d.x_bf16;
        C = d.colonnes;
        N = d.n;
        xq += tranche * blockIdx.y;
        xs = xq + uint64_t(mma_n_pad(N)) * C;
    }
    const uint32_t B = C / 32u;
    const uint32_t w = blockIdx.x * 8u + (threadIdx.x >> 5), voie = threadIdx.x & 31u;
    if (w >= N * B) return;
    const uint32_t n = w / B, b = w % B;
    const uint64_t i = uint64_t(n) * C + 32u * b + voie;
    const float v = bf16 ? __uint_as_float(uint32_t(static_cast<const uint16_t*>(x)[i]) << 16) : static_cast<const float*>(x)[i];
    float m = fabsf(v);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, d));
    int E = -127;
    if (m > 0.0f) {
        const int em = int((__float_as_uint(m) >> 23) & 255u) - 127;  // floor(log2 m) (subnormals: -127)
        E = max(-127, min(127, em - 8));
    }
    const float q = v * __uint_as_float(uint32_t(127 - E) << 23);  // x / 2^E, exact (|E| <= 127)
    uint16_t paire;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(paire) : "f"(0.0f), "f"(q));
    const uint32_t kp = voie < 16u ? 2u * voie : 2u * (voie - 16u) + 1u;
    xq[uint64_t(n) * C + 32u * b + kp] = uint8_t(paire & 0xFFu);
    if (voie == 0) xs[uint64_t(n) * B + b] = uint8_t(E + 127);
}

bool gemm_mxfp4_possible(uint32_t C, uint32_t N) { return mma_smem(N, C, 3u) <= 220u * 1024u; }

uint64_t gemm_mxfp4_espace(uint32_t C, uint32_t N) { return uint64_t(mma_n_pad(N)) * C + uint64_t(mma_n_pad(N)) * (C / 32u); }

cudaError_t lancer_gemm_mxfp4(const uint8_t* codes, const uint8_t* ech, const float* biais, const void* x, uint32_t x_bf16,
                              float* y, uint32_t R, uint32_t C, uint32_t N, uint8_t* espace, uint32_t* erreur,
                              cudaStream_t flux) {
    uint8_t* xq = espace;
    uint8_t* xs = espace + uint64_t(mma_n_pad(N)) * C;
    const uint32_t B = C / 32u;
    cudaError_t e = lancer_pdl(k_quantifier_mxfp8, dim3((N * B + 7u) / 8u), dim3(256), 0, flux, x, x_bf16, C, N, xq, xs,
                               static_cast<const DescGemm*>(nullptr), uint64_t(0));
    if (e != cudaSuccess) return e;
    const uint32_t E = mma_etages(N, C), smem = mma_smem(N, C, E);
    if ((e = assurer_smem(reinterpret_cast<const void*>(k_gemm_mxfp4), int(smem))) != cudaSuccess) return e;
    ArgsMma a{codes, ech, biais, xq, xs, y, R, C, N, erreur};
    return lancer_pdl(k_gemm_mxfp4, dim3((R + MMA_M - 1) / MMA_M), dim3(MMA_FILS), smem, flux, a,
                      static_cast<const DescGemm*>(nullptr), static_cast<uint8_t*>(nullptr), uint64_t(0), E);
}

// A batch of nb matrices (descriptors on the device; rows, columns and tokens at most
// lignes_max, colonnes_max, n_max): one launch quantizes every matrix's x into its workspace
// slice, one launch runs every matrix's row tiles (grid y = the matrix).
cudaError_t lancer_gemm_mxfp4_lot(const DescGemm* descs, uint32_t nb, uint32_t lignes_max, uint32_t colonnes_max,
                                  uint32_t n_max, uint8_t* espace, uint32_t* erreur, cudaStream_t flux) {
    const uint64_t tranche = (gemm_mxfp4_espace(colonnes_max, n_max) + 255u) & ~uint64_t(255);
    const uint32_t B = colonnes_max / 32u;
    cudaError_t e = lancer_pdl(k_quantifier_mxfp8, dim3((n_max * B + 7u) / 8u, nb), dim3(256), 0, flux,
                               static_cast<const void*>(nullptr), 0u, colonnes_max, n_max, espace,
                               static_cast<uint8_t*>(nullptr), descs, tranche);
    if (e != cudaSuccess) return e;
    const uint32_t E = mma_etages(n_max, colonnes_max), smem = mma_smem(n_max, colonnes_max, E);
    if ((e = assurer_smem(reinterpret_cast<const void*>(k_gemm_mxfp4), int(smem))) != cudaSuccess) return e;
    ArgsMma a{};
    a.erreur = erreur;
    return lancer_pdl(k_gemm_mxfp4, dim3((lignes_max + MMA_M - 1) / MMA_M, nb), dim3(MMA_FILS), smem, flux, a, descs,
                      espace, tranche, E);
}

uint64_t gemm_mxfp4_lot_espace(uint32_t colonnes_max, uint32_t n_max, uint32_t nb) {
    return uint64_t(nb) * ((gemm_mxfp4_espace(colonnes_max, n_max) + 255u) & ~uint64_t(255));
}

}  // namespace tb
