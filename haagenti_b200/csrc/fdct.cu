// Factored DCT-III: the IDCT along one axis as a pack pass plus two short
// tensor-core DFT stages (the stages run on dft_stage_kernel, idct_gemm.cu).
//
// For a row c[0..L) (L even, H = L/2 = P*Q) the orthonormal DCT-III
// x[n] = sum_k alpha(k) c[k] cos(pi (2n+1) k / 2L) is computed as
//   pack   : Z[k] = (V[k] + V[k+H]) + i (V[k] - V[k+H]) e^{2 pi i k / L},  k < H,
//            V[k] = w_k (c'[k] - i c'[L-k]) e^{i pi k / 2L},  w_0 = 1, w_k = 1/2,
//            c'[0] = c[0]/sqrt(2), c'[L] = 0            (Makhoul's reordering
//            of the DCT into a length-L real IDFT, halved into a length-H
//            complex IDFT of the even/odd samples)
//   stage 1: G[m1][k2] = e^{2 pi i k2 m1 / H} sum_k1 e^{2 pi i k1 m1 / P} Z[Q k1 + k2]
//   stage 2: z[m1 + P m2] = sum_k2 e^{2 pi i k2 m2 / Q} G[m1][k2]
//   output : x[4j] = Re z[j], x[4j+2] = Im z[j]                 (j < H/2)
//            x[4(H-1-j)+3] = Re z[j], x[4(H-1-j)+1] = Im z[j]   (j >= H/2)
//            times sqrt(2/L).
// The same transform as haagenti_core::dct::idct_1d's inverse Makhoul
// (crates/haagenti-core/src/dct.rs:154-259), factored so that the two DFTs
// are dense P- and Q-point complex matrix products on tcgen05 instead of an
// FFT.  Each pass reads and writes fp16 rows; the layouts are chosen so that
// every pass reads and writes contiguous memory:
//   pack    c rows [b][n]            -> Z  [b][k2][k1][re,im]
//   stage 1 Z  rows (b, k2), K=2P   -> G  [m1][b][k2][re,im]  (twiddled)
//   stage 2 G  rows (m1, b), K=2Q   -> Y  [n][b]              (transposed)
// so two applications (rows, then the rows of the transposed result) give
// the 2-D transform X = A_M F A_N^T with the output in row-major order.
// The folded forms (stage modes 4-6, idct_gemm.cu) change the layouts:
//   mode 4: Z [k2][b][k1] (the pack's k2_major output), stage 1 with the
//           twiddle in per-k2 matrices -> G [m1][k2][re,im][b];
//   mode 6: no Z at all where 64 <= 2P <= 128: the lines stored as
//           T'[b][k2][r] = x[Q r + k2] (the spectral pack's TR output, or the
//           previous pass's transposed output with its lines in the slot
//           order of line_slot) and stage 1 with the Makhoul coefficients
//           and the twiddle in per-(k2, Q - k2) matrices -> the same G;
//   mode 5: stage 2 reading G as an MN-major operand -> Y [n][b].
//
// The pack is written with the combined coefficients
//   alpha_k = w_k' e^{i pi k / 2L} (1 + i e^{2 pi i k / L}),  w_0' = 1/sqrt(2), w_k' = 1/2
//   beta_k  = 1/2 e^{i pi (k+H) / 2L} (1 - i e^{2 pi i k / L})
//   Z[k]    = alpha_k (c[k] - i c[L-k]) + beta_k (c[H+k] - i c[H-k])
// (one float4 per k, computed once per length in f64).
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "common.cuh"

namespace hct {
namespace {

__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }

// Shared-memory index of row element k: 8 fp16 (16 bytes) of padding after
// every 64 elements and SPAD2 more after every 512.  Every group of 8
// elements stays 16-byte aligned (the row is staged and expanded with
// 16-byte stores), and the pack's reads are free of bank conflicts: a warp
// reads 8 consecutive elements (5 words at most) at 4 places 8 Q elements
// apart, which are 8 banks apart with SPAD2 = 16 for Q = 64 (296 words) and
// SPAD2 = 8 for Q = 128 (584 words).
__host__ __device__ __forceinline__ constexpr uint32_t spad2_of(int qc) { return qc == 64 ? 16 : 8; }

template <int QC>
__host__ __device__ __forceinline__ uint32_t spad(uint32_t k) {
    return k + 8 * (k >> 6) + spad2_of(QC) * (k >> 9);
}

// staged row: L elements, padding, and the zero c[L] at spad(L)
__host__ __device__ __forceinline__ uint32_t srow_halves(uint32_t L, int qc) {
    return L + 8 * (L >> 6) + spad2_of(qc) * (L >> 9) + 8;
}

__device__ __forceinline__ uint32_t pack_z(float re, float im) {
    const __half2 h = __floats2half2_rn(re, im);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// spad<QC>(Q (K + j) + x) - spad<QC>(Q K + x) for a compile-time Q = QC in {64, 128}:
// Q K a multiple of 512 and 0 <= x < Q (no 512-boundary inside a run other
// than the one at Q j = 512), and likewise spad(M - x - Q j) =
// spad(M - x) - koff(j) below a multiple M of 512 with 1 <= x <= Q / 2.
template <int QC>
__device__ __forceinline__ constexpr uint32_t koff(int j) {
    return (uint32_t)(QC * j + 8 * ((QC * j) / 64) + spad2_of(QC) * ((QC * j) / 512));
}

// 32 bytes at a 32-byte aligned global address in one access (sm_100)
__device__ __forceinline__ void st_global_v8(uint32_t *p, const uint32_t (&v)[8]) {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(v[0]),
                 "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}

// Output slot of line b: b itself, or, when the next pass folds the Makhoul
// pack into its stage 1 (stage mode 6), (b mod pq) p2 + b / pq for that
// pass's factors pq = Q and p2 = 2P, so that its lines read
// T'[n][k2][r] = x[Q r + k2] as whole 2P-value columns.
__device__ __forceinline__ uint64_t line_slot(uint64_t b, uint32_t pq, uint32_t p2) {
    return pq ? (b % pq) * p2 + b / pq : b;
}

__device__ __forceinline__ float ld_h(const uint16_t *s, uint32_t i) {
    return __half2float(__ushort_as_half(s[i]));
}

// One lane's share of the pack: row k2 in [1, Q/2] and the run of J
// consecutive k1 = J g .. J g + J - 1.  For each k = Q k1 + k2 of the run it
// reads a = c[k], b = c[L-k], c = c[H+k], d = c[H-k] and writes
//   Z[k]   = alpha_k (a - i b) + beta_k (c - i d)
//   Z[H-k] = w [conj(alpha_k) (d - i c) + conj(beta_k) (a + i b)],
//            w = e^{i pi / 4}
// (alpha_{H-k} = w conj(alpha_k) and beta_{H-k} = w^3 conj(beta_k) for
// k != 0, so the table is read once per pair).  Z[H-k] lies in row Q - k2
// at k1' = P - 1 - k1: two runs of J contiguous outputs.  The row k2 = Q/2 is
// its own partner row; its runs write only Z[k], which covers it.
// The coefficients of a run follow from those of its first k by recurrence:
// with u = e^{i pi k / 2L} and v = e^{i 5 pi k / 2L} (k >= 1),
//   alpha_k = (u + i v) / 2,   beta_k = e^{i pi / 4} (u - i v) / 2,
// and k -> k + Q multiplies u by rot.(x, y) = e^{i pi Q / 2L} and v by
// rot.(z, w) = e^{i 5 pi Q / 2L}; u and v of the first k are recovered from its
// table entry, so a run of J outputs loads one float4 instead of J.  REC
// selects that recurrence (fewer L1 wavefronts, for the L1-bound column pack)
// or one table load per k (fewer instructions, for the issue-bound row pack
// that also decodes the payload).
template <int QC, int J, bool REC>
__device__ __forceinline__ void pack_run(const uint16_t *s, const float4 *__restrict__ coef,
                                         float4 rot, uint32_t L, uint32_t P, uint32_t Q,
                                         uint32_t g, uint32_t k2, uint32_t *__restrict__ orow,
                                         uint64_t ks) {
    constexpr float RS2 = 0.70710678118654752440f;
    constexpr float RS2H = 0.35355339059327376220f;  // sqrt(2) / 4
    const uint32_t H = L / 2, k1a = J * g;
    const uint32_t ka = Q * k1a + k2;  // k of the run's first element
    const float4 t0 = coef[ka];
    // gamma = e^{-i pi / 4} beta;  u = alpha + gamma,  v = -i (alpha - gamma)
    const float gr = RS2 * (t0.z + t0.w), gi = RS2 * (t0.w - t0.z);
    float ur = t0.x + gr, ui = t0.y + gi, vr = t0.y - gi, vi = gr - t0.x;
    uint32_t *zd = orow + (uint64_t)k2 * ks + k1a;
    uint32_t *yd = orow + (uint64_t)(Q - k2) * ks + (P - J - k1a);
    const bool partner = 2 * k2 != Q;
    const uint32_t pa = spad<QC>(ka), pb = spad<QC>(L - ka), pc = spad<QC>(H + ka), pd = spad<QC>(H - ka);
    uint32_t zo[J], yo[J];
#pragma unroll
    for (int h = 0; h < J / 4; h++) {
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int j = 4 * h + t;
            uint32_t ia, ib, ic, id;
            if (QC) {
                ia = pa + koff<QC>(j);
                ib = pb - koff<QC>(j);
                ic = pc + koff<QC>(j);
                id = pd - koff<QC>(j);
            } else {
                const uint32_t k = ka + Q * (uint32_t)j;
                ia = spad<QC>(k);
                ib = spad<QC>(L - k);
                ic = spad<QC>(H + k);
                id = spad<QC>(H - k);
            }
            const float a = ld_h(s, ia), b = ld_h(s, ib), c = ld_h(s, ic), d = ld_h(s, id);
            float4 tt;  // (alpha.re, alpha.im, beta.re, beta.im) of k
            if (!REC) {
                tt = coef[ka + Q * (uint32_t)j];
            } else {
                const float x = ur + vi, y = ui - vr;
                tt = make_float4(0.5f * (ur - vi), 0.5f * (ui + vr), RS2H * (x - y), RS2H * (x + y));
                const float nur = ur * rot.x - ui * rot.y, nvr = vr * rot.z - vi * rot.w;
                ui = ur * rot.y + ui * rot.x;
                vi = vr * rot.w + vi * rot.z;
                ur = nur;
                vr = nvr;
            }
            zo[j] = pack_z(fmaf(tt.x, a, fmaf(tt.y, b, fmaf(tt.z, c, tt.w * d))),
                           fmaf(tt.y, a, fmaf(-tt.x, b, fmaf(tt.w, c, -tt.z * d))));
            const float s1 = d + c, s2 = d - c, s3 = a - b, s4 = a + b;
            // Z[H - k] goes to position J - 1 - j of the partner run
            yo[J - 1 - j] = pack_z(RS2 * fmaf(tt.x, s1, fmaf(tt.y, s2, fmaf(tt.z, s3, tt.w * s4))),
                                   RS2 * fmaf(tt.x, s2, fmaf(-tt.y, s1, fmaf(tt.z, s4, -tt.w * s3))));
        }
    }
    if (J == 8) {
        // runs of 8 start at multiples of 8 words (P % 8 == 0): 32-byte aligned
        st_global_v8(zd, reinterpret_cast<const uint32_t(&)[8]>(zo));
        if (partner) st_global_v8(yd, reinterpret_cast<const uint32_t(&)[8]>(yo));
    } else {
#pragma unroll
        for (int v = 0; v < J / 4; v++) {
            reinterpret_cast<uint4 *>(zd)[v] =
                make_uint4(zo[4 * v], zo[4 * v + 1], zo[4 * v + 2], zo[4 * v + 3]);
            if (partner)
                reinterpret_cast<uint4 *>(yd)[v] =
                    make_uint4(yo[4 * v], yo[4 * v + 1], yo[4 * v + 2], yo[4 * v + 3]);
        }
    }
}

// Row k2 = 0 pairs with itself at k1' = P - k1: its outputs are computed
// directly, one k1 per lane (k = 0 reads c[L], the zero at spad<QC>(L)).
template <int QC>
__device__ __forceinline__ void pack_k2_zero(const uint16_t *s, const float4 *__restrict__ coef,
                                             uint32_t L, uint32_t Q, uint32_t k1,
                                             uint32_t *__restrict__ orow) {
    const uint32_t H = L / 2, k = Q * k1;
    const float a = ld_h(s, spad<QC>(k)), b = ld_h(s, spad<QC>(L - k));
    const float c = ld_h(s, spad<QC>(H + k)), d = ld_h(s, spad<QC>(H - k));
    const float4 tt = coef[k];
    orow[k1] = pack_z(fmaf(tt.x, a, fmaf(tt.y, b, fmaf(tt.z, c, tt.w * d))),
                      fmaf(tt.y, a, fmaf(-tt.x, b, fmaf(tt.w, c, -tt.z * d))));
}

// Pack of one staged row s (spad layout) into its output row, in (k2, k1)
// order, by the warps warp, warp + nwarps, ...
//   QC in {64, 128} (runs of 8): warp task (kg, og) takes rows
//     k2 = 8 kg + 1 .. 8 kg + 8 and runs g = 4 og .. 4 og + 3, lane
//     8 o + r taking row 8 kg + 1 + r and run 4 og + o: the 4 runs of a row
//     are 128 contiguous output bytes, so a 16-byte store of the warp
//     touches 8 rows;
//   QC = 0 (any Q, runs of 4): lane items (run g, row k2), k2 fastest;
// the remaining tasks cover row k2 = 0.
template <int QC, int J, bool REC>
__device__ __forceinline__ void pack_row(const uint16_t *s, const float4 *__restrict__ coef,
                                         float4 rot, uint32_t L, uint32_t P, uint32_t Q,
                                         uint32_t *__restrict__ orow, uint64_t ks, uint32_t warp,
                                         uint32_t nwarps, uint32_t lane) {
    const uint32_t half = QC ? (uint32_t)QC / 2 : Q / 2;
    const uint32_t runs = P / J;
    uint32_t ntask;
    if (QC) ntask = (half / 8) * ((runs + 3) / 4);
    else ntask = (runs * half + 31) / 32;
    const uint32_t nall = ntask + (P + 31) / 32;
    for (uint32_t tau = warp; tau < nall; tau += nwarps) {
        if (tau < ntask) {
            if (QC) {
                const uint32_t kg = tau % (half / 8), og = tau / (half / 8);
                const uint32_t g = 4 * og + (lane >> 3);
                if (g < runs)
                    pack_run<QC, J, REC>(s, coef, rot, L, P, QC, g, 8 * kg + 1 + (lane & 7), orow, ks);
            } else {
                const uint32_t i = 32 * tau + lane;
                if (i < runs * half) {
                    const uint32_t g = i / half;
                    pack_run<0, J, REC>(s, coef, rot, L, P, Q, g, 1 + i - g * half, orow, ks);
                }
            }
        } else {
            const uint32_t k1 = 32 * (tau - ntask) + lane;
            if (k1 < P) pack_k2_zero<QC>(s, coef, L, QC ? (uint32_t)QC : Q, k1, orow);
        }
    }
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// Pack of dense fp16 rows (stride ld_in): one CTA per row at a time, several
// CTAs per SM; the row is staged with 16-byte cp.async copies.
template <int THREADS, int QC, int J>
__global__ void __launch_bounds__(THREADS, THREADS == 128 ? 7 : 3) makhoul_pack_kernel(
    const uint16_t *__restrict__ in, uint64_t ld_in, uint64_t B, uint32_t L, uint32_t P,
    uint32_t Q, const float4 *__restrict__ coef, float4 rot, uint32_t *__restrict__ out,
    uint64_t bs, uint64_t ks, uint32_t pq, uint32_t p2) {
    extern __shared__ uint4 smem_v[];
    uint16_t *srow = reinterpret_cast<uint16_t *>(smem_v);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool vec = ((ld_in & 7) == 0) && (((uintptr_t)in & 15) == 0);
    const uint32_t nv = L / 8;  // L % 32 == 0 for every factored length
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(srow);
    if (threadIdx.x == 0) srow[spad<QC>(L)] = 0;  // c[L] = 0 (never overwritten)
    for (uint64_t b = blockIdx.x; b < B; b += gridDim.x) {
        __syncthreads();  // previous row fully consumed
        const uint16_t *row = in + b * ld_in;
        if (vec) {
            for (uint32_t v = threadIdx.x; v < nv; v += THREADS)
                cp_async16(sbase + 2 * spad<QC>(8 * v), row + 8 * v);
            cp_async_wait_all();
        } else {
            for (uint32_t k = threadIdx.x; k < L; k += THREADS) srow[spad<QC>(k)] = row[k];
        }
        __syncthreads();
        pack_row<QC, J, true>(srow, coef, rot, L, P, Q, out + line_slot(b, pq, p2) * bs, ks,
                              warp, THREADS / 32, lane);
    }
}

// Pack for P that is not a multiple of 4 (the vocabulary lengths, e.g.
// H = 16000 = 125 x 128 or 64128 = 501 x 128): the output row of each
// (b, k2) is padded to Pp = round_up(P, 8) complex values (zeros past P), so
// that stage 1 reads 16-byte aligned rows of K = 2 Pp.  Each thread writes 4
// consecutive k1 of one k2 (one 16-byte store) and computes every Z[k] from
// its four inputs (no partner sharing: the partner of a run is not an aligned
// run when P % 4 != 0).  The inputs are read from global memory (a row of up
// to 2^20 elements, cached in L1/L2): consecutive threads take consecutive
// k2, so each of the four reads of a warp is contiguous.
__global__ void __launch_bounds__(256) makhoul_pack_generic_kernel(
    const uint16_t *__restrict__ in, uint64_t ld_in, uint64_t B, uint32_t L, uint32_t P,
    uint32_t Pp, uint32_t Q, const float4 *__restrict__ coef, uint32_t *__restrict__ out,
    uint64_t bs, uint64_t ks, uint32_t pq, uint32_t p2) {
    const uint32_t H = L / 2, runs = Pp / 4;
    const uint64_t items = (uint64_t)runs * Q;
    for (uint64_t b = blockIdx.y; b < B; b += gridDim.y) {
        const uint16_t *row = in + b * ld_in;
        uint32_t *orow = out + line_slot(b, pq, p2) * bs;
        for (uint64_t it = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; it < items;
             it += (uint64_t)gridDim.x * blockDim.x) {
            const uint32_t g = (uint32_t)(it / Q), k2 = (uint32_t)(it - (uint64_t)g * Q);
            uint32_t z[4];
#pragma unroll
            for (int t = 0; t < 4; t++) {
                const uint32_t k1 = 4 * g + t;
                z[t] = 0;
                if (k1 < P) {
                    const uint32_t k = Q * k1 + k2;
                    const float a = ld_h(row, k), bb = k ? ld_h(row, L - k) : 0.0f;
                    const float c = ld_h(row, H + k), d = ld_h(row, H - k);
                    const float4 tt = coef[k];
                    z[t] = pack_z(fmaf(tt.x, a, fmaf(tt.y, bb, fmaf(tt.z, c, tt.w * d))),
                                  fmaf(tt.y, a, fmaf(-tt.x, bb, fmaf(tt.w, c, -tt.z * d))));
                }
            }
            *reinterpret_cast<uint4 *>(orow + (uint64_t)k2 * ks + 4 * g) =
                make_uint4(z[0], z[1], z[2], z[3]);
        }
    }
}

// Row pack straight from the spectral payload (bitmap ++ INT4): one CTA per
// row at a time, several CTAs per SM.
//   A. the row's 64-bit bitmap words into shared memory and their
//      popcounts scanned over the CTA (each word's rank within the row);
//      warp 0 reads the row's first rank from the rank directory of
//      launch_spectral_rank plus a partial popcount;
//   B. the row's coefficients in rank order are staged: when the row has at
//      most L/2 of them as fp16 (nibble - 8) * scale, 8 ranks per thread and
//      step (a nibble placed in the mantissa of 1024.0 gives 1024 + nibble;
//      HSUB2 of 1032 is exact and HMUL2 rounds the exact product once, as
//      the f32 product rounded to fp16 does); else the raw nibble bytes and
//      the f32 scales;
//   C. lane l of a warp step takes byte (l & 7) of word 4 s + (l >> 3) and
//      writes its 8 elements (zero where the bit is clear) as one 16-byte
//      store into the staged row;
//   D. pack_row.
// Requires L % 64 == 0 (rows start on a 64-bit bitmap boundary).
__host__ __device__ __forceinline__ uint32_t spack_raw_nib_bytes(uint32_t L) {
    return (L / 2 + 16 + 15) & ~15u;
}

// bytes of the staging area: L/2 + 16 fp16 values, or L/2 nibble bytes
// (+ slack) and L/32 + 4 f32 scales
__host__ __device__ __forceinline__ uint32_t spack_stage_bytes(uint32_t L) {
    const uint32_t vals = L + 32, raw = spack_raw_nib_bytes(L) + (L / 32 + 4) * 4;
    return vals > raw ? vals : raw;
}

__host__ __device__ __forceinline__ uint32_t spack_words_pad(uint32_t L) {
    return (L / 64 + 3) & ~3u;
}

__host__ __device__ __forceinline__ size_t spack_smem_bytes(uint32_t L, int qc) {
    return (size_t)srow_halves(L, qc) * 2 + (size_t)spack_words_pad(L) * 12 +
           spack_stage_bytes(L);
}

// Transposed staging of the TR variant (output for stage mode 6): Q rows
// (k2) of tr_pitch(P) fp16 (r), 16-byte chunk c of row k2 at chunk
// c ^ ((k2 >> 3) & 7), so that the expand's 2-byte stores (8 lanes at k2
// 8 apart) and the copy-out's 16-byte loads are free of bank conflicts.
#ifndef SPACK_TR_CTAS
#define SPACK_TR_CTAS 8  // resident CTAs per SM of the 128-thread TR variant (<= 64 registers)
#endif
__host__ __device__ __forceinline__ uint32_t tr_pitch(uint32_t P) {
    return (2 * P + 63) / 64 * 64 + 8;
}
__host__ __device__ __forceinline__ size_t spack_tr_smem_bytes(uint32_t L, uint32_t P, uint32_t Q) {
    return (size_t)Q * tr_pitch(P) * 2 + (size_t)spack_words_pad(L) * 12 + spack_stage_bytes(L);
}

// 16 bits of the nibble section at byte nb (even); bytes at or past nib_len
// read as zero
__device__ __forceinline__ uint32_t ld_nib16(const uint8_t *nibbles, uint32_t nb,
                                             uint64_t nib_len) {
    if ((uint64_t)nb + 1 < nib_len) return *reinterpret_cast<const uint16_t *>(nibbles + nb);
    return (uint64_t)nb < nib_len ? (uint32_t)nibbles[nb] : 0u;
}

__device__ __forceinline__ uint16_t deq_nibble_h(uint32_t byte, uint32_t r, float scale) {
    const uint32_t nib = (r & 1) ? byte >> 4 : byte & 0xfu;
    return __half_as_ushort(__float2half_rn(__fmul_rn((float)((int)nib - 8), scale)));
}

// TR: instead of the pack, each line is written transposed, out[slot][k2][r]
// = c[Q r + k2] (Q % 8 == 0, 2P <= 128), the input of stage mode 6 (which
// folds the Makhoul pack into its matrices); steps C and D become
//   C'. the staging (pitch TRP = tr_pitch(P), a compile-time 72 or 136) is
//       cleared with 16-byte stores; then the set bits of a byte (one r,
//       k2 .. k2 + 7) store their values into it, clear bits store nothing;
//   D'. the staging is copied out as 16-byte chunks of the contiguous
//       2 P Q-value output line.
template <int THREADS, int QC, int J, int TRP>
__global__ void __launch_bounds__(THREADS, THREADS == 128 ? (TRP ? SPACK_TR_CTAS : 6) : 2)
    spectral_pack_kernel(
    const uint8_t *__restrict__ payload, uint64_t bmb, const uint32_t *__restrict__ chunk_base,
    uint64_t group_off, const uint64_t *__restrict__ meta, uint64_t B, uint32_t L, uint32_t P,
    uint32_t Q, const float4 *__restrict__ coef, float4 rot, uint32_t *__restrict__ out,
    uint64_t bs, uint64_t ks, uint32_t pq, uint32_t p2) {
    constexpr uint32_t NW = THREADS / 32;
    constexpr bool TR = TRP != 0;
    extern __shared__ uint4 smem_v[];
    __shared__ uint32_t warp_tot[NW];
    __shared__ uint32_t s_rank0;
    const uint32_t W = L / 64;
    uint16_t *srow = reinterpret_cast<uint16_t *>(smem_v);
    const int qsh = (Q & (Q - 1)) == 0 ? __ffs(Q) - 1 : -1;  // log2 Q, or -1
    uint64_t *sw = reinterpret_cast<uint64_t *>(srow + (TR ? Q * (uint32_t)TRP : srow_halves(L, QC)));
    uint32_t *swr = reinterpret_cast<uint32_t *>(sw + spack_words_pad(L));
    uint8_t *stage = reinterpret_cast<uint8_t *>(swr + spack_words_pad(L));
    uint16_t *vals_s = reinterpret_cast<uint16_t *>(stage);
    uint8_t *nib_s = stage;
    float *sc_s = reinterpret_cast<float *>(stage + spack_raw_nib_bytes(L));
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint64_t k_total = meta[0];
    const uint64_t nib_len = (k_total + 1) >> 1;  // bytes of the nibble section
    const uint8_t *scales = payload + bmb;
    const uint8_t *nibbles = payload + meta[1];
    const bool bad = meta[2] != 0;
    const uint64_t *bm64 = reinterpret_cast<const uint64_t *>(payload);
    const uint32_t *bm32 = reinterpret_cast<const uint32_t *>(payload);
    const uint32_t wpt = (W + THREADS - 1) / THREADS, w0 = tid * wpt;
    // expand geometry of this lane: byte (lane & 7) of word (lane >> 3) of a span
    const uint32_t sub = lane >> 3, bsh = 8 * (lane & 7);
    const uint64_t below8 = (1ull << bsh) - 1ull;
    if (!TR && tid == 0) srow[spad<QC>(L)] = 0;  // c[L] = 0 (never overwritten)

    for (uint64_t b = blockIdx.x; b < B; b += gridDim.x) {
        __syncthreads();  // previous row fully consumed
        if (TR) {
            // C'. (first half) the staging reads zero where no bit is set
            for (uint32_t i = tid; i < Q * (uint32_t)TRP / 8; i += THREADS)
                reinterpret_cast<uint4 *>(srow)[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        // A. bitmap words and their ranks
        uint32_t cnt = 0;
        for (uint32_t i = 0; i < wpt; i++) {
            const uint32_t w = w0 + i;
            if (w < W) {
                const uint64_t x = bm64[b * W + w];
                sw[w] = x;
                cnt += __popcll(x);
            }
        }
        uint32_t incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= (uint32_t)o) incl += t;
        }
        if (lane == 31) warp_tot[warp] = incl;
        if (warp == 0) {
            const uint64_t word0 = b * (uint64_t)(L / 32);
            const uint64_t c0 = word0 / 32;  // its 1024-bit chunk
            uint32_t part = 0;
            for (uint64_t w = c0 * 32 + lane; w < word0; w += 32) part += __popc(bm32[w]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
            if (lane == 0)
                s_rank0 = chunk_base[c0] + chunk_base[group_off + c0 / RANK_GROUP] + part;
        }
        __syncthreads();
        uint32_t run = incl - cnt, row_count = 0;
#pragma unroll
        for (uint32_t v = 0; v < NW; v++) {
            const uint32_t t = warp_tot[v];
            run += v < warp ? t : 0u;
            row_count += t;
        }
        for (uint32_t i = 0; i < wpt; i++) {
            const uint32_t w = w0 + i;
            if (w < W) {
                swr[w] = run;
                run += __popcll(sw[w]);
            }
        }
        const uint32_t rank0 = s_rank0;
        const bool packed = 2 * row_count <= L;
        const uint32_t a8 = rank0 & ~7u;  // vals_s[i] holds rank a8 + i
        const uint32_t nb0 = rank0 >> 1, sb0 = rank0 >> 5;
        // B. stage the row's coefficients (rank order); a short payload
        // (meta[2]) decodes to zeros and never reads past its end
        if (!bad) {
            if (packed) {
                const uint32_t n8 = (rank0 + row_count - a8 + 7) >> 3;
                const __half2 off = __float2half2_rn(1032.0f);
                for (uint32_t gi = tid; gi < n8; gi += THREADS) {
                    const uint32_t r = a8 + 8 * gi;  // below k_total
                    const uint32_t nb = r >> 1;      // a multiple of 4
                    const uint32_t x =
                        ld_nib16(nibbles, nb, nib_len) | (ld_nib16(nibbles, nb + 2, nib_len) << 16);
                    const uint32_t e = x & 0x0F0F0F0Fu, o = (x >> 4) & 0x0F0F0F0Fu;
                    const __half sh = __ushort_as_half(
                        *reinterpret_cast<const uint16_t *>(scales + 2 * (r >> 5)));
                    const __half2 s2 = __halves2half2(sh, sh);
                    uint32_t wv[4];
#pragma unroll
                    for (uint32_t i = 0; i < 4; i++) {
                        // (nibble 2i, nibble 2i + 1) as (1024 + n0, 1024 + n1)
                        const uint32_t p = (__byte_perm(e, o, i | ((4 + i) << 8)) & 0x00FF00FFu) |
                                           0x64006400u;
                        const __half2 h = __hmul2(__hsub2(*reinterpret_cast<const __half2 *>(&p), off), s2);
                        wv[i] = *reinterpret_cast<const uint32_t *>(&h);
                    }
                    *reinterpret_cast<uint4 *>(vals_s + 8 * gi) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                }
            } else {
                const uint32_t nb1 = (rank0 + row_count + 1) >> 1;
                const uint32_t sb1 = row_count ? ((rank0 + row_count - 1) >> 5) + 1 : sb0;
                for (uint32_t i = nb0 + tid; i < nb1; i += THREADS) nib_s[i - nb0] = nibbles[i];
                for (uint32_t i = sb0 + tid; i < sb1; i += THREADS)
                    sc_s[i - sb0] = __half2float(__ushort_as_half(
                        (uint16_t)((uint32_t)scales[2 * (uint64_t)i] |
                                   ((uint32_t)scales[2 * (uint64_t)i + 1] << 8))));
            }
        }
        __syncthreads();
        // C. expand the words into the staged row, 4 words per warp step
        const uint32_t roff = rank0 - a8;
        for (uint32_t sp = warp; 4 * sp < W; sp += NW) {
            const uint32_t w = 4 * sp + sub;
            if (w < W) {
                const uint64_t x = sw[w];
                const uint32_t byte = bad ? 0u : (uint32_t)(x >> bsh) & 0xffu;
                const uint32_t q = swr[w] + __popcll(x & below8);  // rank within the row
                if (TR) {
                    // elements n0 .. n0 + 7: one r, k2 = k20 .. k20 + 7
                    const uint32_t n0 = 64 * w + 8 * (lane & 7);
                    const uint32_t rr = qsh >= 0 ? n0 >> qsh : n0 / Q;
                    const uint32_t k20 = n0 - rr * Q;
                    uint16_t *d = srow + k20 * (uint32_t)TRP + 8 * ((rr >> 3) ^ ((k20 >> 3) & 7)) +
                                  (rr & 7);
                    if (packed) {
                        uint32_t r = q + roff;
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            if ((byte >> t) & 1u) d[t * TRP] = vals_s[r++];
                        }
                    } else {
                        uint32_t gr = rank0 + q;
#pragma unroll
                        for (int t = 0; t < 8; t++) {
                            if ((byte >> t) & 1u) {
                                d[t * TRP] = deq_nibble_h(nib_s[(gr >> 1) - nb0], gr,
                                                          sc_s[(gr >> 5) - sb0]);
                                gr++;
                            }
                        }
                    }
                    continue;
                }
                uint32_t h[8];
                if (packed) {
                    uint32_t r = q + roff;
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const uint32_t bit = (byte >> t) & 1u;
                        h[t] = bit ? (uint32_t)vals_s[r] : 0u;
                        r += bit;
                    }
                } else {
                    uint32_t gr = rank0 + q;
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        const uint32_t bit = (byte >> t) & 1u;
                        h[t] = bit ? (uint32_t)deq_nibble_h(nib_s[(gr >> 1) - nb0], gr,
                                                            sc_s[(gr >> 5) - sb0])
                                   : 0u;
                        gr += bit;
                    }
                }
                *reinterpret_cast<uint4 *>(srow + spad<QC>(64 * w + 8 * (lane & 7))) =
                    make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16),
                               h[6] | (h[7] << 16));
            }
        }
        __syncthreads();
        if (TR) {
            // D'. line slot: Q rows of 2P values, contiguous.  A warp step
            // copies 32 / cp2 rows, lane (sub-row, chunk c) with cp2 the power
            // of two >= the row's cpr 16-byte chunks (8 or 16)
            const uint32_t cpr = 2 * P / 8;
            const uint32_t csh = cpr > 8 ? 4 : 3, sr = lane >> csh, c = lane & ((1u << csh) - 1);
            uint4 *dst = reinterpret_cast<uint4 *>(out + line_slot(b, pq, p2) * bs);
            if (c < cpr) {
                for (uint32_t k2 = warp * (32u >> csh) + sr; k2 < Q; k2 += NW * (32u >> csh))
                    dst[k2 * cpr + c] = *reinterpret_cast<const uint4 *>(
                        srow + k2 * (uint32_t)TRP + 8 * (c ^ ((k2 >> 3) & 7)));
            }
        } else {
            pack_row<QC, J, false>(srow, coef, rot, L, P, Q, out + line_slot(b, pq, p2) * bs, ks,
                                   warp, NW, lane);
        }
    }
}

// coef[k] = (alpha_k, beta_k) for k < L/2 (see the file comment), in f64.
__global__ void pack_tables_kernel(uint32_t L, float4 *coef) {
    const uint32_t H = L / 2;
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x) {
        double sa, ca, sb, cb, st, ct;
        sincospi((double)k / (2.0 * (double)L), &sa, &ca);          // e^{i pi k / 2L}
        sincospi((double)(k + H) / (2.0 * (double)L), &sb, &cb);    // e^{i pi (k+H) / 2L}
        sincospi(2.0 * (double)k / (double)L, &st, &ct);            // t = e^{2 pi i k / L}
        const double w = k == 0 ? 0.70710678118654752440 : 0.5;
        // alpha = w a (1 + i t) = w a (1 - st + i ct)
        const double pr = 1.0 - st, pi_ = ct;
        const double ar = w * (ca * pr - sa * pi_), ai = w * (ca * pi_ + sa * pr);
        // beta = 1/2 b (1 - i t) = 1/2 b (1 + st - i ct)
        const double qr = 1.0 + st, qi = -ct;
        const double br = 0.5 * (cb * qr - sb * qi), bi = 0.5 * (cb * qi + sb * qr);
        coef[k] = make_float4((float)ar, (float)ai, (float)br, (float)bi);
    }
}

// Realified DFT matrix, K-major, for the B operand of a stage:
// row 2m   = [ cos(2 pi m k / n), -sin(2 pi m k / n) ] over k (interleaved),
// row 2m+1 = [ sin(2 pi m k / n),  cos(2 pi m k / n) ].
// Rows and columns beyond 2n are zero (ld = padded K).
__global__ void dft_matrix_kernel(uint32_t n, uint32_t rows_pad, uint32_t ld, uint16_t *out) {
    const uint32_t total = rows_pad * ld;
    for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += gridDim.x * blockDim.x) {
        const uint32_t r = idx / ld, c = idx - r * ld;
        float v = 0.0f;
        if (r < 2 * n && c < 2 * n) {
            const uint32_t m = r >> 1, k = c >> 1;
            const uint32_t j = (uint32_t)(((uint64_t)m * k) % n);
            double s, co;
            sincospi(2.0 * (double)j / (double)n, &s, &co);
            if ((r & 1) == 0) v = (c & 1) == 0 ? (float)co : (float)-s;
            else v = (c & 1) == 0 ? (float)s : (float)co;
        }
        out[idx] = f2h(v);
    }
}

// Per-k2 stage-1 matrices with the twiddle folded in (mode 4 of the stage
// kernel): entry (k2, o = 2 m1 + ri, k = 2 k1 + rk) is the realified
// e^{2 pi i m1 (Q k1 + k2) / H} (rows [cos, -sin], [sin, cos] as in
// dft_matrix_kernel), the angle reduced exactly in integers and evaluated in f64.
__global__ void twiddled_dft_kernel(uint32_t P, uint32_t Q, uint32_t w_rows, uint32_t ld,
                                    uint16_t *out) {
    const uint64_t H = (uint64_t)P * Q;
    const uint64_t per_k2 = (uint64_t)w_rows * ld, total = per_k2 * Q;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t k2 = idx / per_k2, rem = idx - k2 * per_k2;
        const uint32_t o = (uint32_t)(rem / ld), k = (uint32_t)(rem - (uint64_t)o * ld);
        float v = 0.0f;
        if (o < 2 * P && k < 2 * P) {
            const uint64_t m1 = o >> 1, k1 = k >> 1;
            const uint64_t j = (m1 * (Q * k1 + k2)) % H;
            double sn, cs;
            sincospi(2.0 * (double)j / (double)H, &sn, &cs);
            if ((o & 1) == 0) v = (k & 1) == 0 ? (float)cs : (float)-sn;
            else v = (k & 1) == 0 ? (float)sn : (float)cs;
        }
        out[idx] = f2h(v);
    }
}

// Per-pair stage-1 matrices of stage mode 6: the Makhoul pack and the
// twiddle folded into stage 1.  That stage reads, for 128 lines n and a pair
// u in [0, Q/2], columns u and (Q - u) mod Q of T'[n][k2][r] = x[Q r + k2]
// (x the line of length L = 2H, H = P Q), each as kbc k-blocks of 64 values
// (K = 128 kbc; the values past r = 2P read as zero).  Rows 0..127 (half
// h = 0) give G[m1][k2] for k2 = u, rows 128..255 (h = 1) for k2 = Q - u
// (zero for u = 0 and u = Q/2, whose pair has one k2):
//   G[m1][k2] = sum_k1 e^{2 pi i m1 k / H} Z[k],  k = Q k1 + k2,
//   Z[k] = alpha_k (a - i b) + beta_k (c - i d),
//   a = x[k], b = x[L - k], c = x[H + k], d = x[H - k]   (x[L] = 0),
// alpha_k and beta_k as in pack_tables_kernel.  The four inputs sit at
//   a: column k2, r = k1            c: column k2, r = P + k1
//   b: column C,  r = 2P - 1 - k1   d: column C,  r = P - 1 - k1   (C = Q - k2, k2 >= 1)
//   b: column 0,  r = 2P - k1 (k1 >= 1)   d: column 0, r = P - k1  (k2 = 0)
// where the k2 of the half is in block h of K and C in the other block.
// Entry (u, 128 h + 2 m1 + ri, 64 kbc blk + r) is the real (ri = 0) or
// imaginary (ri = 1) part of the complex coefficient of that real input,
// evaluated in f64 and rounded once to fp16.
__global__ void makhoul_fold_kernel(uint32_t P, uint32_t Q, uint32_t kbc, uint16_t *out) {
    const uint64_t H = (uint64_t)P * Q, L = 2 * H;
    const uint32_t K = 128 * kbc, KC = 64 * kbc;
    const uint64_t per_u = 256ull * K, total = per_u * (Q / 2 + 1);
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t u = (uint32_t)(idx / per_u);
        const uint32_t rem = (uint32_t)(idx - (uint64_t)u * per_u);
        const uint32_t row = rem / K, kk = rem - row * K;
        const uint32_t h = row >> 7, m1 = (row & 127) >> 1, ri = row & 1;
        const uint32_t blk = kk / KC, r = kk - blk * KC;
        double v = 0.0;
        if (m1 < P && r < 2 * P && (h == 0 || (u != 0 && 2 * u != Q))) {
            const uint32_t k2 = h ? Q - u : u;
            int role = -1;  // 0 a, 1 b, 2 c, 3 d
            uint32_t k1 = 0;
            if (blk == h) {
                role = r < P ? 0 : 2;
                k1 = r < P ? r : r - P;
            } else if (k2 != 0) {
                role = r < P ? 3 : 1;
                k1 = r < P ? P - 1 - r : 2 * P - 1 - r;
            } else if (r != 0) {
                role = r <= P ? 3 : 1;
                k1 = r <= P ? P - r : 2 * P - r;
            }
            if (role >= 0) {
                const uint64_t k = (uint64_t)Q * k1 + k2;
                double cr, ci;
                if (role <= 1) {
                    // alpha = w e^{i pi k / 2L} (1 + i t), t = e^{2 pi i k / L}
                    double sa, ca, st, ct;
                    sincospi((double)k / (2.0 * (double)L), &sa, &ca);
                    sincospi(2.0 * (double)k / (double)L, &st, &ct);
                    const double w = k == 0 ? 0.70710678118654752440 : 0.5;
                    const double pr = 1.0 - st, pi_ = ct;
                    cr = w * (ca * pr - sa * pi_);
                    ci = w * (ca * pi_ + sa * pr);
                } else {
                    // beta = 1/2 e^{i pi (k + H) / 2L} (1 - i t)
                    double sb, cb, st, ct;
                    sincospi((double)(k + H) / (2.0 * (double)L), &sb, &cb);
                    sincospi(2.0 * (double)k / (double)L, &st, &ct);
                    const double qr = 1.0 + st, qi = -ct;
                    cr = 0.5 * (cb * qr - sb * qi);
                    ci = 0.5 * (cb * qi + sb * qr);
                }
                if (role == 1 || role == 3) {  // times -i
                    const double t = cr;
                    cr = ci;
                    ci = -t;
                }
                const uint64_t j = ((uint64_t)m1 * k) % H;
                double sn, cs;
                sincospi(2.0 * (double)j / (double)H, &sn, &cs);
                v = ri ? cs * ci + sn * cr : cs * cr - sn * ci;
            }
        }
        out[idx] = __half_as_ushort(__double2half(v));
    }
}

// e^{2 pi i j / H} for j < H, complex fp32 (re, im).
__global__ void twiddle_table_kernel(uint32_t H, float2 *out) {
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < H; j += gridDim.x * blockDim.x) {
        double s, c;
        sincospi(2.0 * (double)j / (double)H, &s, &c);
        out[j] = make_float2((float)c, (float)s);
    }
}

}  // namespace

uint32_t fdct_padded_p(uint32_t P) { return P % 4 == 0 ? P : (P + 7) / 8 * 8; }

bool fdct_factor(uint64_t L, uint32_t *P, uint32_t *Q) {
    if (L < 16 || (L & 1)) return false;
    const uint64_t H = L / 2;
    if (H > (1ull << 31)) return false;
    uint32_t best_p = 0, best_q = 0;
    auto fast_q = [](uint64_t q) { return q == 16 || q == 32 || q == 64 || q == 128; };
    for (uint32_t p = 4; p <= 128; p += 4) {
        if (H % p) continue;
        const uint64_t q = H / p;
        if (q > 128 || q % 4) continue;
        // most balanced split; among equally balanced ones, a Q that the
        // pack kernels specialise (16, 32, 64, 128)
        const uint64_t cur = best_p ? (best_p > best_q ? best_p - best_q : best_q - best_p) : ~0ull;
        const uint64_t d = p > q ? p - q : q - p;
        if (d < cur || (d == cur && fast_q(q) && !fast_q(best_q))) {
            best_p = p;
            best_q = (uint32_t)q;
        }
    }
    if (!best_p) {
        // no split into two multiples of 4 up to 128 (e.g. H = 16000 = 125 x 128 or
        // 64128 = 501 x 128): the largest Q (a multiple of 4, <= 128) dividing H,
        // P = H / Q of any size (stage 1 pads P, and takes the dense-tile
        // contraction beyond 128)
        for (uint32_t q = 128; q >= 4; q -= 4) {
            if (H % q == 0 && H / q <= FDCT_MAX_P) {
                best_q = q;
                best_p = (uint32_t)(H / q);
                break;
            }
        }
        if (!best_p) return false;
    }
    *P = best_p;
    *Q = best_q;
    return true;
}

namespace {

// Specialisation of the pack for (P, Q): runs of 8 with compile-time read
// offsets for Q in {64, 128} and P % 8 == 0; else 0 (runs of 4, any Q).
int pack_qc(uint32_t P, uint32_t Q) {
    if (P % 8 == 0 && (Q == 64 || Q == 128)) return (int)Q;
    return 0;
}

using MakhoulFn = void (*)(const uint16_t *, uint64_t, uint64_t, uint32_t, uint32_t, uint32_t,
                           const float4 *, float4, uint32_t *, uint64_t, uint64_t, uint32_t,
                           uint32_t);
using SpectralFn = void (*)(const uint8_t *, uint64_t, const uint32_t *, uint64_t,
                            const uint64_t *, uint64_t, uint32_t, uint32_t, uint32_t,
                            const float4 *, float4, uint32_t *, uint64_t, uint64_t, uint32_t,
                            uint32_t);

// (e^{i pi Q / 2L}, e^{i 5 pi Q / 2L}): the steps of u and v along k1 (pack_run)
float4 pack_rot(uint32_t L, uint32_t Q) {
    const double a = M_PI * (double)Q / (2.0 * (double)L);
    return make_float4((float)std::cos(a), (float)std::sin(a), (float)std::cos(5.0 * a),
                       (float)std::sin(5.0 * a));
}

template <int T>
MakhoulFn makhoul_fn(int qc) {
    switch (qc) {
        case 64: return makhoul_pack_kernel<T, 64, 8>;
        case 128: return makhoul_pack_kernel<T, 128, 8>;
        default: return makhoul_pack_kernel<T, 0, 4>;
    }
}

template <int T>
SpectralFn spectral_fn(int qc) {
    switch (qc) {
        case 64: return spectral_pack_kernel<T, 64, 8, 0>;
        case 128: return spectral_pack_kernel<T, 128, 8, 0>;
        default: return spectral_pack_kernel<T, 0, 4, 0>;
    }
}

// grid of a row kernel: one CTA per row, so that the block scheduler keeps
// the SMs balanced when other streams' kernels hold some of them (the
// kernels also loop over rows, for grids capped below the row count)
template <typename F>
cudaError_t row_grid(F kern, int threads, size_t smem, uint64_t B, unsigned *grid) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const uint64_t cap = 0x7fffffffull;
    *grid = (unsigned)(B < cap ? (B < 1 ? 1 : B) : cap);
    return cudaSuccess;
}

}  // namespace

cudaError_t launch_makhoul_pack(const half_bits *d_in, uint64_t ld_in, uint64_t B, uint32_t L,
                                uint32_t P, uint32_t Q, const float *d_tables, half_bits *d_out,
                                bool k2_major, uint32_t perm_q, uint32_t perm_2p, cudaStream_t s) {
    if ((uint64_t)P * Q != L / 2 || Q % 4 || L % 8) return cudaErrorInvalidValue;
    if (perm_q && (uint64_t)perm_q * perm_2p != B) return cudaErrorInvalidValue;
    const uint64_t Pp = fdct_padded_p(P);
    // Z[b][k2][k1] (b stride Q Pp, k2 stride Pp) or Z[k2][b][k1] (Pp, B Pp)
    const uint64_t bs = k2_major ? Pp : (uint64_t)Q * Pp, ks = k2_major ? B * Pp : Pp;
    if (P % 4) {
        if ((uintptr_t)d_out & 15) return cudaErrorInvalidValue;
        const uint64_t items = (uint64_t)(fdct_padded_p(P) / 4) * Q;
        const unsigned gx = (unsigned)std::min<uint64_t>((items + 255) / 256, 64);
        const unsigned gy = (unsigned)std::min<uint64_t>(B, 65535);
        makhoul_pack_generic_kernel<<<dim3(gx, gy), 256, 0, s>>>(
            d_in, ld_in, B, L, P, fdct_padded_p(P), Q, reinterpret_cast<const float4 *>(d_tables),
            reinterpret_cast<uint32_t *>(d_out), bs, ks, perm_q, perm_2p);
        return cudaGetLastError();
    }
    if (L % 32) return cudaErrorInvalidValue;
    // the specialised pack writes 32-byte runs: it needs a 32-byte aligned output
    const int qc = ((uintptr_t)d_out & 31) ? 0 : pack_qc(P, Q);
    const size_t smem = (size_t)srow_halves(L, qc) * 2;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const bool small = L <= 16384;
    const int threads = small ? 128 : 256;
    MakhoulFn kern = small ? makhoul_fn<128>(qc) : makhoul_fn<256>(qc);
    unsigned g = 0;
    cudaError_t e = row_grid(kern, threads, smem, B, &g);
    if (e != cudaSuccess) return e;
    kern<<<g, threads, smem, s>>>(d_in, ld_in, B, L, P, Q,
                                  reinterpret_cast<const float4 *>(d_tables), pack_rot(L, Q),
                                  reinterpret_cast<uint32_t *>(d_out), bs, ks, perm_q, perm_2p);
    return cudaGetLastError();
}

bool spectral_pack_supported(uint64_t L) {
    uint32_t P = 0, Q = 0;
    return L % 64 == 0 && L <= (1u << 20) && spack_smem_bytes((uint32_t)L, 64) <= 200 * 1024 &&
           fdct_factor(L, &P, &Q) && P % 4 == 0;
}

cudaError_t launch_spectral_pack(const uint8_t *d_payload, uint64_t bmb, const uint32_t *d_chunk,
                                 const uint64_t *d_meta, uint64_t B, uint32_t L, uint32_t P,
                                 uint32_t Q, const float *d_tables, half_bits *d_out,
                                 bool k2_major, uint32_t perm_q, uint32_t perm_2p,
                                 cudaStream_t s, bool transposed) {
    if (!spectral_pack_supported(L) || (uint64_t)P * Q != L / 2 || P % 4 || Q % 4)
        return cudaErrorInvalidValue;
    if (perm_q && (uint64_t)perm_q * perm_2p != B) return cudaErrorInvalidValue;
    if (transposed) {
        // lines of L values (16-byte aligned), Q a multiple of 8, 2P <= 128
        if (Q % 8 || 2 * P > 128 || ((uintptr_t)d_out & 15)) return cudaErrorInvalidValue;
        const size_t smem = spack_tr_smem_bytes(L, P, Q);
        if (smem > 200 * 1024) return cudaErrorInvalidValue;
        const bool small = L <= 16384;
        const int threads = small ? 128 : 256;
        const bool narrow = tr_pitch(P) == 72;  // 2P <= 64; else 136
        SpectralFn kern = small ? (narrow ? spectral_pack_kernel<128, 0, 4, 72>
                                          : spectral_pack_kernel<128, 0, 4, 136>)
                                : (narrow ? spectral_pack_kernel<256, 0, 4, 72>
                                          : spectral_pack_kernel<256, 0, 4, 136>);
        unsigned g = 0;
        cudaError_t e = row_grid(kern, threads, smem, B, &g);
        if (e != cudaSuccess) return e;
        kern<<<g, threads, smem, s>>>(d_payload, bmb, d_chunk, rank_group_offset(B * (uint64_t)L),
                                      d_meta, B, L, P, Q, reinterpret_cast<const float4 *>(d_tables),
                                      pack_rot(L, Q), reinterpret_cast<uint32_t *>(d_out), L / 2, 0,
                                      perm_q, perm_2p);
        return cudaGetLastError();
    }
    const uint64_t bs = k2_major ? P : (uint64_t)Q * P, ks = k2_major ? B * P : P;
    const int qc = ((uintptr_t)d_out & 31) ? 0 : pack_qc(P, Q);
    const size_t smem = spack_smem_bytes(L, qc);
    const bool small = L <= 16384;
    const int threads = small ? 128 : 256;
    SpectralFn kern = small ? spectral_fn<128>(qc) : spectral_fn<256>(qc);
    unsigned g = 0;
    cudaError_t e = row_grid(kern, threads, smem, B, &g);
    if (e != cudaSuccess) return e;
    kern<<<g, threads, smem, s>>>(d_payload, bmb, d_chunk, rank_group_offset(B * (uint64_t)L),
                                  d_meta, B, L, P, Q, reinterpret_cast<const float4 *>(d_tables),
                                  pack_rot(L, Q), reinterpret_cast<uint32_t *>(d_out), bs, ks,
                                  perm_q, perm_2p);
    return cudaGetLastError();
}

cudaError_t launch_pack_tables(uint32_t L, uint32_t P, uint32_t Q, float *d_tables,
                               cudaStream_t s) {
    if ((uint64_t)P * Q != L / 2) return cudaErrorInvalidValue;
    pack_tables_kernel<<<(L / 2 + 255) / 256, 256, 0, s>>>(L, reinterpret_cast<float4 *>(d_tables));
    return cudaGetLastError();
}

cudaError_t launch_dft_matrix(uint32_t n, uint32_t rows_pad, uint32_t ld, half_bits *d_out,
                              cudaStream_t s) {
    const uint32_t total = rows_pad * ld;
    dft_matrix_kernel<<<(total + 255) / 256, 256, 0, s>>>(n, rows_pad, ld, d_out);
    return cudaGetLastError();
}

cudaError_t launch_twiddled_dft_table(uint32_t P, uint32_t Q, uint32_t w_rows, uint32_t ld,
                                      half_bits *d_out, cudaStream_t s) {
    const uint64_t total = (uint64_t)Q * w_rows * ld;
    const uint64_t g = std::min<uint64_t>((total + 255) / 256, 148ull * 64);
    twiddled_dft_kernel<<<(unsigned)g, 256, 0, s>>>(P, Q, w_rows, ld, d_out);
    return cudaGetLastError();
}

cudaError_t launch_makhoul_fold_table(uint32_t P, uint32_t Q, uint32_t kbc, half_bits *d_out,
                                      cudaStream_t s) {
    if (kbc < 1 || kbc > 2 || 2 * P > 64 * kbc || Q % 2) return cudaErrorInvalidValue;
    const uint64_t total = 256ull * 128 * kbc * (Q / 2 + 1);
    const uint64_t g = std::min<uint64_t>((total + 255) / 256, 148ull * 32);
    makhoul_fold_kernel<<<(unsigned)g, 256, 0, s>>>(P, Q, kbc, d_out);
    return cudaGetLastError();
}

cudaError_t launch_twiddle_table(uint32_t H, float *d_out, cudaStream_t s) {
    twiddle_table_kernel<<<(H + 255) / 256, 256, 0, s>>>(H, reinterpret_cast<float2 *>(d_out));
    return cudaGetLastError();
}

}  // namespace hct
