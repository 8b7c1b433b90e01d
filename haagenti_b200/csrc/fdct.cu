// Factored DCT-III: the IDCT along one axis as a pack pass plus two short
// tensor-core DFT stages (the stages run on umma_gemm_kernel, modes 2 and 3).
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
#include <cuda_fp16.h>

#include <cmath>

#include "common.cuh"

namespace hct {
namespace {

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }

// Shared-memory index of row element k: two fp16 of padding every 64
// elements, so reads at stride Q (a multiple of 4) spread over the banks.
__device__ __forceinline__ uint32_t pad_idx(uint32_t k) { return k + 2 * (k >> 6); }

// Shared-memory word index of Z[k] in the transpose buffer (one pad word per
// 64 words, so the stride-Q reads of the output phase spread over the banks).
__device__ __forceinline__ uint32_t zpad_idx(uint32_t k) { return k + (k >> 6); }

// One CTA per row (grid-stride over the batch), three phases:
//  1. the row is staged in shared memory (fp16, coalesced 16-byte loads);
//  2. Z[k] for k < H is computed in natural order (c[k], c[L-k], c[H+k],
//     c[H-k]; twiddle ta[k] = e^{i pi k / 2L} read coalesced; e^{i pi (k+H)/2L}
//     = ta[k] e^{i pi/4}; e^{2 pi i k / L} = ta[k]^4) into a second buffer;
//  3. Z is written out in (k2, k1) order, k = Q k1 + k2, k1 fastest, one warp
//     per k2 row, as 4-byte fp16 pairs.
__global__ void __launch_bounds__(512) makhoul_pack_kernel(const uint16_t *__restrict__ in,
                                                           uint64_t ld_in, uint64_t B, uint32_t L,
                                                           uint32_t P, uint32_t Q,
                                                           const float2 *__restrict__ ta,
                                                           const float2 *__restrict__ tb,
                                                           uint32_t *__restrict__ out) {
    extern __shared__ uint16_t srow[];
    const uint32_t H = L / 2;
    uint32_t *zbuf = reinterpret_cast<uint32_t *>(srow + ((pad_idx(L) + 8) & ~7u));
    const float inv_sqrt2 = 0.70710678118654752440f;
    const float c45 = 0.70710678118654752440f;  // e^{i pi/4} = (c45, c45)
    const bool vec = ((ld_in & 7) == 0) && (((uintptr_t)in & 15) == 0) && ((L & 7) == 0);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    (void)tb;
    for (uint64_t b = blockIdx.x; b < B; b += gridDim.x) {
        const uint16_t *row = in + b * ld_in;
        __syncthreads();  // previous row fully consumed
        if (vec) {
            // 8 independent 16-byte loads in flight per thread before any store
            const uint4 *r4 = reinterpret_cast<const uint4 *>(row);
            const uint32_t nv = L / 8;
            for (uint32_t v0 = threadIdx.x; v0 < nv; v0 += 8 * blockDim.x) {
                uint4 x[8];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const uint32_t v = v0 + u * blockDim.x;
                    if (v < nv) x[u] = r4[v];
                }
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const uint32_t v = v0 + u * blockDim.x;
                    if (v < nv) {
                        // 8 elements never straddle a 64-element pad
                        uint32_t *d = reinterpret_cast<uint32_t *>(srow + pad_idx(8 * v));
                        d[0] = x[u].x;
                        d[1] = x[u].y;
                        d[2] = x[u].z;
                        d[3] = x[u].w;
                    }
                }
            }
        } else {
            for (uint32_t k = threadIdx.x; k < L; k += blockDim.x) srow[pad_idx(k)] = row[k];
        }
        __syncthreads();
        for (uint32_t k = threadIdx.x; k < H; k += blockDim.x) {
            float ck = h2f(srow[pad_idx(k)]);
            float cLk = 0.0f, w = 1.0f;
            if (k == 0) {
                ck *= inv_sqrt2;
            } else {
                cLk = h2f(srow[pad_idx(L - k)]);
                w = 0.5f;
            }
            const float cHk = h2f(srow[pad_idx(H + k)]);
            const float cHmk = h2f(srow[pad_idx(H - k)]);  // H - k >= 1 for k < H
            const float2 a = ta[k];
            const float2 bb = make_float2(c45 * (a.x - a.y), c45 * (a.x + a.y));
            const float2 a2 = make_float2(a.x * a.x - a.y * a.y, 2.0f * a.x * a.y);
            const float2 t = make_float2(a2.x * a2.x - a2.y * a2.y, 2.0f * a2.x * a2.y);
            // V[k] = w (ck - i cLk) e^{i pi k / 2L}
            const float vr = w * (ck * a.x + cLk * a.y);
            const float vi = w * (ck * a.y - cLk * a.x);
            // U = V[k+H] = 1/2 (cHk - i cHmk) e^{i pi (k+H) / 2L}
            const float ur = 0.5f * (cHk * bb.x + cHmk * bb.y);
            const float ui = 0.5f * (cHk * bb.y - cHmk * bb.x);
            // Z = (V + U) + i (V - U) e^{2 pi i k / L}
            const float dr = vr - ur, di = vi - ui;
            const float er = dr * t.x - di * t.y, ei = dr * t.y + di * t.x;
            zbuf[zpad_idx(k)] =
                (uint32_t)f2h((vr + ur) - ei) | ((uint32_t)f2h((vi + ui) + er) << 16);
        }
        __syncthreads();
        uint32_t *orow = out + b * (uint64_t)H;
        for (uint32_t k2 = warp; k2 < Q; k2 += nwarps)
            for (uint32_t k1 = lane; k1 < P; k1 += 32)
                orow[k2 * P + k1] = zbuf[zpad_idx(Q * k1 + k2)];
    }
}

// ta[k] = e^{i pi k / 2L} for k < L; tb[k] = e^{2 pi i k / L} for k < L/2.
__global__ void pack_tables_kernel(uint32_t L, float2 *ta, float2 *tb) {
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < L; k += gridDim.x * blockDim.x) {
        double s, c;
        sincospi((double)k / (2.0 * (double)L), &s, &c);
        ta[k] = make_float2((float)c, (float)s);
        if (k < L / 2) {
            sincospi(2.0 * (double)k / (double)L, &s, &c);
            tb[k] = make_float2((float)c, (float)s);
        }
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

// e^{2 pi i j / H} for j < H, complex fp32 (re, im).
__global__ void twiddle_table_kernel(uint32_t H, float2 *out) {
    for (uint32_t j = blockIdx.x * blockDim.x + threadIdx.x; j < H; j += gridDim.x * blockDim.x) {
        double s, c;
        sincospi(2.0 * (double)j / (double)H, &s, &c);
        out[j] = make_float2((float)c, (float)s);
    }
}

}  // namespace

bool fdct_factor(uint64_t L, uint32_t *P, uint32_t *Q) {
    if (L < 16 || (L & 1)) return false;
    const uint64_t H = L / 2;
    uint32_t best_p = 0, best_q = 0;
    for (uint32_t p = 4; p <= 128; p += 4) {
        if (H % p) continue;
        const uint64_t q = H / p;
        if (q > 128 || q % 4) continue;
        // most balanced split
        const uint64_t cur = best_p ? (best_p > best_q ? best_p - best_q : best_q - best_p) : ~0ull;
        const uint64_t d = p > q ? p - q : q - p;
        if (d < cur) { best_p = p; best_q = (uint32_t)q; }
    }
    if (!best_p) return false;
    *P = best_p;
    *Q = best_q;
    return true;
}

cudaError_t launch_makhoul_pack(const half_bits *d_in, uint64_t ld_in, uint64_t B, uint32_t L,
                                uint32_t P, uint32_t Q, const float *d_tables, half_bits *d_out,
                                cudaStream_t s) {
    // row (fp16, padded) + Z transpose buffer (u32, padded)
    const size_t row_elems = ((size_t)L + 2 * (L / 64) + 8 + 7) & ~(size_t)7;
    const size_t smem = row_elems * sizeof(uint16_t) + ((size_t)L / 2 + L / 128 + 8) * 4;
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(makhoul_pack_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    uint64_t g = B < 148ull * 8 ? B : 148ull * 8;
    if (g < 1) g = 1;
    const float2 *ta = reinterpret_cast<const float2 *>(d_tables);
    makhoul_pack_kernel<<<(unsigned)g, 512, smem, s>>>(d_in, ld_in, B, L, P, Q, ta, ta + L,
                                                       reinterpret_cast<uint32_t *>(d_out));
    return cudaGetLastError();
}

cudaError_t launch_pack_tables(uint32_t L, float *d_tables, cudaStream_t s) {
    float2 *ta = reinterpret_cast<float2 *>(d_tables);
    pack_tables_kernel<<<(L + 255) / 256, 256, 0, s>>>(L, ta, ta + L);
    return cudaGetLastError();
}

cudaError_t launch_dft_matrix(uint32_t n, uint32_t rows_pad, uint32_t ld, half_bits *d_out,
                              cudaStream_t s) {
    const uint32_t total = rows_pad * ld;
    dft_matrix_kernel<<<(total + 255) / 256, 256, 0, s>>>(n, rows_pad, ld, d_out);
    return cudaGetLastError();
}

cudaError_t launch_twiddle_table(uint32_t H, float *d_out, cudaStream_t s) {
    twiddle_table_kernel<<<(H + 255) / 256, 256, 0, s>>>(H, reinterpret_cast<float2 *>(d_out));
    return cudaGetLastError();
}

}  // namespace hct
