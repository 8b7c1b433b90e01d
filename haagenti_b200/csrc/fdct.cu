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
//
// The pack is written with the combined coefficients
//   alpha_k = w_k' e^{i pi k / 2L} (1 + i e^{2 pi i k / L}),  w_0' = 1/sqrt(2), w_k' = 1/2
//   beta_k  = 1/2 e^{i pi (k+H) / 2L} (1 - i e^{2 pi i k / L})
//   Z[k]    = alpha_k (c[k] - i c[L-k]) + beta_k (c[H+k] - i c[H-k])
// (one float4 per k, computed once per length in f64).
#include <cuda_fp16.h>

#include <cmath>

#include "common.cuh"

namespace hct {
namespace {

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }

// Shared-memory index of row element k: two fp16 of padding every 64
// elements, so the pack's reads at stride Q (lanes = consecutive k1) spread
// over the banks.
__device__ __forceinline__ uint32_t pad_idx(uint32_t k) { return k + 2 * (k >> 6); }

__host__ __device__ __forceinline__ uint32_t srow_halves(uint32_t L) {
    return (L + 2 * (L >> 6) + 8) & ~7u;
}

__device__ __forceinline__ uint32_t pack_z(float re, float im) {
    const __half2 h = __floats2half2_rn(re, im);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Pack of one staged row, written straight to the output row in (k2, k1)
// order, k = Q k1 + k2: warp w takes the k2 rows w, w + nwarps, ... <= Q/2 and
// lane l the k1 = l, l + 32, ...; each item also produces its partner H - k,
// which reads the same four inputs c[k], c[L-k], c[H+k], c[H-k] with the
// roles permuted and lies at k2' = Q - k2, k1' = P - 1 - k1 (k2 > 0) or
// k2' = 0, k1' = P - k1 (k2 = 0).  coefT holds (alpha_k, beta_k) in the same
// (k2, k1) order, so every global access of a warp is contiguous.
// srow[pad_idx(L)] must hold zero: it is c[L] of the k = 0 term.  Along a
// lane's k1 = l, l + 32, ... every index moves by a constant (32 Q is a
// multiple of 64, so pad_idx(k + 32 Q) = pad_idx(k) + 33 Q).
// The same pack for NR rows staged sstride halves apart (outputs ostride
// words apart, the first nvalid of them written): the coefficient loads and
// the index arithmetic are shared by the rows.
template <int NR>
__device__ __forceinline__ void pack_rows(const uint16_t *srow, uint32_t sstride,
                                          const float4 *__restrict__ coefT, uint32_t L, uint32_t P,
                                          uint32_t Q, uint32_t *__restrict__ orow, uint64_t ostride,
                                          uint32_t nvalid) {
    const uint32_t H = L / 2;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const uint32_t sstep = 33 * Q;
    for (uint32_t k2 = warp; 2 * k2 <= Q; k2 += nwarps) {
        const uint32_t k1_end = k2 == 0 ? P / 2 + 1 : (2 * k2 == Q ? P / 2 : P);
        const uint32_t k = Q * lane + k2;
        uint32_t ia = pad_idx(k), ib = pad_idx(L - k), ic = pad_idx(H + k), id = pad_idx(H - k);
        uint32_t io = k2 * P + lane;
        uint32_t jo = k2 == 0 ? P - lane : (Q - k2) * P + (P - 1 - lane);
        for (uint32_t k1 = lane; k1 < k1_end; k1 += 32) {
            const float4 t = coefT[io];  // (alpha.re, alpha.im, beta.re, beta.im)
            const bool partner = k2 != 0 || (k1 != 0 && 2 * k1 != P);  // k != 0 and k != H/2
            const float4 u = partner ? coefT[jo] : t;
#pragma unroll
            for (int q = 0; q < NR; q++) {
                const uint16_t *sr = srow + q * sstride;
                const float ck = h2f(sr[ia]);
                const float cLk = h2f(sr[ib]);
                const float cHk = h2f(sr[ic]);
                const float cHmk = h2f(sr[id]);  // H - k >= 1 for k < H
                const float zr = fmaf(t.x, ck, fmaf(t.y, cLk, fmaf(t.z, cHk, t.w * cHmk)));
                const float zi = fmaf(t.y, ck, fmaf(-t.x, cLk, fmaf(t.w, cHk, -t.z * cHmk)));
                if ((uint32_t)q < nvalid) orow[q * ostride + io] = pack_z(zr, zi);
                if (partner && (uint32_t)q < nvalid) {
                    // k' = H - k: c[k'] = c[H-k], c[L-k'] = c[H+k], c[H+k'] = c[L-k], c[H-k'] = c[k]
                    const float yr = fmaf(u.x, cHmk, fmaf(u.y, cHk, fmaf(u.z, cLk, u.w * ck)));
                    const float yi = fmaf(u.y, cHmk, fmaf(-u.x, cHk, fmaf(u.w, cLk, -u.z * ck)));
                    orow[q * ostride + jo] = pack_z(yr, yi);
                }
            }
            ia += sstep;
            ib -= sstep;
            ic += sstep;
            id -= sstep;
            io += 32;
            jo -= 32;
        }
    }
}

__device__ __forceinline__ void pack_row(const uint16_t *srow, const float4 *__restrict__ coefT,
                                         uint32_t L, uint32_t P, uint32_t Q,
                                         uint32_t *__restrict__ orow) {
    const uint32_t H = L / 2;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    const uint32_t sstep = 33 * Q;
    for (uint32_t k2 = warp; 2 * k2 <= Q; k2 += nwarps) {
        const uint32_t k1_end = k2 == 0 ? P / 2 + 1 : (2 * k2 == Q ? P / 2 : P);
        if (lane >= k1_end) continue;
        const uint32_t k = Q * lane + k2;
        const uint16_t *pa = srow + pad_idx(k), *pb = srow + pad_idx(L - k);
        const uint16_t *pc = srow + pad_idx(H + k), *pd = srow + pad_idx(H - k);
        const uint32_t io = k2 * P + lane;
        const uint32_t jo = k2 == 0 ? P - lane : (Q - k2) * P + (P - 1 - lane);
        const float4 *ct = coefT + io, *cu = coefT + jo;
        uint32_t *ot = orow + io, *ou = orow + jo;
        // the partner H - k exists except for k = 0 and k = H/2 (both in row k2 = 0)
        const bool edge = k2 == 0;
        for (uint32_t k1 = lane; k1 < k1_end; k1 += 32) {
            const float ck = h2f(*pa);
            const float cLk = h2f(*pb);
            const float cHk = h2f(*pc);
            const float cHmk = h2f(*pd);  // H - k >= 1 for k < H
            const float4 t = *ct;         // (alpha.re, alpha.im, beta.re, beta.im)
            const float zr = fmaf(t.x, ck, fmaf(t.y, cLk, fmaf(t.z, cHk, t.w * cHmk)));
            const float zi = fmaf(t.y, ck, fmaf(-t.x, cLk, fmaf(t.w, cHk, -t.z * cHmk)));
            *ot = pack_z(zr, zi);
            if (!edge || (k1 != 0 && 2 * k1 != P)) {
                // k' = H - k: c[k'] = c[H-k], c[L-k'] = c[H+k], c[H+k'] = c[L-k], c[H-k'] = c[k]
                const float4 u = *cu;
                const float yr = fmaf(u.x, cHmk, fmaf(u.y, cHk, fmaf(u.z, cLk, u.w * ck)));
                const float yi = fmaf(u.y, cHmk, fmaf(-u.x, cHk, fmaf(u.w, cLk, -u.z * ck)));
                *ou = pack_z(yr, yi);
            }
            pa += sstep;
            pb -= sstep;
            pc += sstep;
            pd -= sstep;
            ct += 32;
            cu -= 32;
            ot += 32;
            ou -= 32;
        }
    }
}

// Pack of dense fp16 rows (stride ld_in): one CTA per NR rows (sharing the
// coefficient loads and index arithmetic), the rows staged in shared memory
// with up to 4 independent 16-byte loads in flight per thread and row.
// THREADS = 256, NR = 2 with 4 CTAs per SM for rows up to 16384 elements;
// THREADS = 512, NR = 1 with 2 beyond (a staged row then takes up to 57 KB).
template <int THREADS, int MIN_CTAS, int NR>
__global__ void __launch_bounds__(THREADS, MIN_CTAS) makhoul_pack_kernel(
    const uint16_t *__restrict__ in, uint64_t ld_in, uint64_t B, uint32_t L, uint32_t P,
    uint32_t Q, const float4 *__restrict__ coefT, uint32_t *__restrict__ out) {
    extern __shared__ uint16_t srow[];
    const uint32_t sstride = srow_halves(L);
    const bool vec = ((ld_in & 7) == 0) && (((uintptr_t)in & 15) == 0) && ((L & 7) == 0);
    const uint32_t nv = L / 8;
    if (threadIdx.x < NR) srow[threadIdx.x * sstride + pad_idx(L)] = 0;  // c[L] = 0
    for (uint64_t b = (uint64_t)blockIdx.x * NR; b < B; b += (uint64_t)gridDim.x * NR) {
        const uint32_t nvalid = (uint32_t)(B - b < (uint64_t)NR ? B - b : (uint64_t)NR);
        __syncthreads();  // previous rows fully consumed
#pragma unroll
        for (int q = 0; q < NR; q++) {
            if ((uint32_t)q >= nvalid) break;
            const uint16_t *row = in + (b + q) * ld_in;
            uint16_t *sr = srow + q * sstride;
            if (vec) {
                const uint4 *r4 = reinterpret_cast<const uint4 *>(row);
                for (uint32_t v0 = threadIdx.x; v0 < nv; v0 += 4 * THREADS) {
                    uint4 x[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const uint32_t v = v0 + u * THREADS;
                        if (v < nv) x[u] = __ldg(r4 + v);
                    }
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const uint32_t v = v0 + u * THREADS;
                        if (v < nv) {  // 8 elements never straddle a 64-element pad
                            uint32_t *d = reinterpret_cast<uint32_t *>(sr + pad_idx(8 * v));
                            d[0] = x[u].x;
                            d[1] = x[u].y;
                            d[2] = x[u].z;
                            d[3] = x[u].w;
                        }
                    }
                }
            } else {
                for (uint32_t k = threadIdx.x; k < L; k += THREADS) sr[pad_idx(k)] = row[k];
            }
        }
        __syncthreads();
        pack_rows<NR>(srow, sstride, coefT, L, P, Q, out + b * (uint64_t)(L / 2), L / 2, nvalid);
    }
}

// Row pack straight from the spectral payload (bitmap ++ INT4).  Each CTA
// decodes the coefficients of its row into shared memory and then runs the
// pack:
//   A. warp w takes a run of the row's 64-bit bitmap words (a multiple of 4,
//      one per lane) and a warp scan of their popcounts; warp 0 adds up the
//      row's rank (the rank directory of launch_spectral_rank for its
//      1024-bit chunk plus a partial popcount);
//   B. the row's coefficients in rank order are staged in shared memory:
//      fp16((nibble - 8) * scale) per set bit, four ranks per thread and
//      step (one 16-bit nibble load, one scale) when the row has at most L/2
//      of them; else the raw nibble bytes and the f32 scales;
//   C. each warp expands its words 256 elements per step: lane l takes bitmap
//      byte l of four consecutive words and writes its 8 elements (zero where
//      the bit is clear) as four 32-bit words, which the one-word pad per 64
//      elements spreads over all 32 banks.
// Requires L % 64 == 0 (rows start on a 64-bit bitmap boundary) and
// L / 64 <= 32 * SPACK_WARPS.
constexpr int SPACK_THREADS = 512;
constexpr int SPACK_WARPS = SPACK_THREADS / 32;

// bytes of the staging area behind the row: L/2 + 8 fp16 values, or L/2
// nibble bytes (+ 16 slack) and L/32 + 4 f32 scales
__host__ __device__ __forceinline__ uint32_t spack_stage_bytes(uint32_t L) {
    const uint32_t vals = L + 16, raw = ((L / 2 + 16 + 15) & ~15u) + (L / 32 + 4) * 4;
    return vals > raw ? vals : raw;
}

__device__ __forceinline__ float deq_nibble(uint32_t byte, uint64_t r, float scale) {
    const uint32_t nib = (r & 1) ? byte >> 4 : byte & 0xfu;
    return __fmul_rn((float)((int)nib - 8), scale);
}

__global__ void __launch_bounds__(SPACK_THREADS, 4) spectral_pack_kernel(
    const uint8_t *__restrict__ payload, uint64_t bmb, const uint32_t *__restrict__ chunk_base,
    uint64_t group_off, const uint64_t *__restrict__ meta, uint64_t B, uint32_t L, uint32_t P,
    uint32_t Q, const float4 *__restrict__ coef, uint32_t *__restrict__ out) {
    extern __shared__ uint16_t srow[];
    __shared__ uint32_t warp_tot[SPACK_WARPS];
    __shared__ uint32_t s_rank_start;
    uint8_t *stage = reinterpret_cast<uint8_t *>(srow + srow_halves(L));
    uint16_t *vals_s = reinterpret_cast<uint16_t *>(stage);
    uint8_t *nib_s = stage;
    float *sc_s = reinterpret_cast<float *>(stage + ((L / 2 + 16 + 15) & ~15u));
    uint32_t *srow32 = reinterpret_cast<uint32_t *>(srow);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t segs = L / 64;
    const uint32_t spw = ((segs + SPACK_WARPS - 1) / SPACK_WARPS + 3) & ~3u;  // <= 32
    const uint32_t seg0 = warp * spw;
    const uint32_t nseg = seg0 < segs ? min(spw, segs - seg0) : 0u;
    const uint64_t k_total = meta[0];
    const uint64_t nib_len = (k_total + 1) >> 1;  // bytes of the nibble section
    const uint8_t *scales = payload + bmb;
    const uint8_t *nibbles = payload + meta[1];
    const bool bad = meta[2] != 0;
    const uint64_t *bm64 = reinterpret_cast<const uint64_t *>(payload);
    const uint32_t *bm32 = reinterpret_cast<const uint32_t *>(payload);
    // expand geometry of this lane: byte (lane & 7) of word (lane >> 3) of a span
    const uint32_t sub = lane >> 3, bshift = 8 * (lane & 7);
    const uint64_t below8 = (1ull << bshift) - 1ull;
    // raw-nibble expand (rows over half full): elements (2l, 2l + 1) of a word
    const uint32_t pair_shift = 2 * lane;
    const uint64_t below2 = (1ull << pair_shift) - 1ull;
    if (threadIdx.x == 0) srow[pad_idx(L)] = 0;  // c[L] = 0 (never overwritten)

    for (uint64_t b = blockIdx.x; b < B; b += gridDim.x) {
        __syncthreads();  // previous row fully consumed
        // A. bitmap words and their ranks
        const uint64_t mw = lane < nseg ? bm64[b * segs + seg0 + lane] : 0ull;
        const uint32_t cnt = __popcll(mw);
        uint32_t incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
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
                s_rank_start = chunk_base[c0] + chunk_base[group_off + c0 / RANK_GROUP] + part;
        }
        __syncthreads();
        // rank of this warp's first bit within the row, and the row's count
        const uint32_t wt = lane < SPACK_WARPS ? warp_tot[lane] : 0u;
        uint32_t wincl = wt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, wincl, o);
            if (lane >= o) wincl += t;
        }
        const uint32_t before = __shfl_sync(0xffffffffu, wincl - wt, warp);
        const uint32_t row_count = __shfl_sync(0xffffffffu, wincl, SPACK_WARPS - 1);
        const uint64_t rank0 = s_rank_start;
        const bool packed_vals = 2 * row_count <= L;
        const uint64_t a4 = rank0 & ~3ull;  // vals_s[i] holds rank a4 + i
        const uint64_t nb0 = rank0 >> 1, sb0 = rank0 >> 5;
        // B. stage the row's coefficients (rank order); a short payload
        // (meta[2]) decodes to zeros and never reads past its end
        if (!bad) {
            if (packed_vals) {
                const uint32_t ngroups = (uint32_t)((rank0 + row_count + 3 - a4) >> 2);
                for (uint32_t g = threadIdx.x; g < ngroups; g += SPACK_THREADS) {
                    const uint64_t r = a4 + 4ull * g;  // a multiple of 4, below k_total
                    const uint64_t nb = r >> 1;        // even: a 16-bit aligned pair
                    uint32_t nib4;
                    if (nb + 1 < nib_len) nib4 = *reinterpret_cast<const uint16_t *>(nibbles + nb);
                    else nib4 = nb < nib_len ? (uint32_t)nibbles[nb] : 0u;
                    const float sc = __half2float(__ushort_as_half(
                        *reinterpret_cast<const uint16_t *>(scales + 2 * (r >> 5))));
                    float v[4];
#pragma unroll
                    for (int t = 0; t < 4; t++)
                        v[t] = __fmul_rn((float)((int)((nib4 >> (4 * t)) & 0xfu) - 8), sc);
                    *reinterpret_cast<uint2 *>(vals_s + 4 * g) =
                        make_uint2(pack_z(v[0], v[1]), pack_z(v[2], v[3]));
                }
            } else {
                const uint64_t nb1 = (rank0 + row_count + 1) >> 1;
                const uint64_t sb1 = row_count ? ((rank0 + row_count - 1) >> 5) + 1 : sb0;
                for (uint64_t i = nb0 + threadIdx.x; i < nb1; i += SPACK_THREADS)
                    nib_s[i - nb0] = nibbles[i];
                for (uint64_t i = sb0 + threadIdx.x; i < sb1; i += SPACK_THREADS)
                    sc_s[i - sb0] = __half2float(__ushort_as_half(
                        (uint16_t)((uint32_t)scales[2 * i] | ((uint32_t)scales[2 * i + 1] << 8))));
            }
        }
        __syncthreads();
        // C. expand this warp's words into the staged row
        const uint32_t wrank = before + incl - cnt;  // rank of my word within the row
        if (packed_vals) {
            const uint32_t roff = (uint32_t)(rank0 - a4);
            uint32_t *dst = srow32 + 33 * (seg0 + sub) + 4 * (lane & 7);
            const uint32_t nspan = (nseg + 3) >> 2;  // nseg <= 32: s stays below 32
            for (uint32_t i = 0; i < nspan; i++, dst += 132) {  // 4 x (64 elements + pad)
                const uint32_t s = 4 * i + sub;
                const uint64_t w = __shfl_sync(0xffffffffu, mw, s);
                const uint32_t wr = __shfl_sync(0xffffffffu, wrank, s);
                if (s < nseg) {
                    const uint32_t byte = bad ? 0u : (uint32_t)(w >> bshift) & 0xffu;
                    uint32_t r = wr + roff + __popcll(w & below8);
                    uint32_t h[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const uint32_t bit = (byte >> j) & 1u;
                        h[j] = bit ? (uint32_t)vals_s[r] : 0u;
                        r += bit;
                    }
                    dst[0] = h[0] | (h[1] << 16);
                    dst[1] = h[2] | (h[3] << 16);
                    dst[2] = h[4] | (h[5] << 16);
                    dst[3] = h[6] | (h[7] << 16);
                }
            }
        } else {
            uint32_t *dst = srow32 + 33 * seg0 + lane;  // 64 elements + 2 pad halves per word
            for (uint32_t i = 0; i < nseg; i++, dst += 33) {
                const uint64_t w = __shfl_sync(0xffffffffu, mw, i);
                const uint32_t r = __shfl_sync(0xffffffffu, wrank, i) + __popcll(w & below2);
                const uint32_t m2 = (uint32_t)(w >> pair_shift) & 3u;
                uint32_t pair = 0;
                if (!bad && m2) {
                    const uint64_t g0 = rank0 + r, g1 = g0 + (m2 & 1u);
                    float v0 = 0.0f, v1 = 0.0f;
                    if (m2 & 1u) v0 = deq_nibble(nib_s[(g0 >> 1) - nb0], g0, sc_s[(g0 >> 5) - sb0]);
                    if (m2 & 2u) v1 = deq_nibble(nib_s[(g1 >> 1) - nb0], g1, sc_s[(g1 >> 5) - sb0]);
                    pair = pack_z(v0, v1);
                }
                *dst = pair;
            }
        }
        __syncthreads();
        pack_row(srow, coef, L, P, Q, out + b * (uint64_t)(L / 2));
    }
}

// coefT[k2 * P + k1] = (alpha_k, beta_k), k = Q k1 + k2 < L/2 (see the file
// comment), in f64.
__global__ void pack_tables_kernel(uint32_t L, uint32_t P, uint32_t Q, float4 *coefT) {
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
        coefT[(k % Q) * P + k / Q] = make_float4((float)ar, (float)ai, (float)br, (float)bi);
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
    const bool small = L <= 16384;
    const size_t smem = (size_t)srow_halves(L) * 2 * (small ? 2 : 1);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    auto kern = small ? makhoul_pack_kernel<256, 4, 2> : makhoul_pack_kernel<512, 2, 1>;
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const uint64_t per_sm = small ? 4 : 2;
    const uint64_t units = small ? (B + 1) / 2 : B;  // row pairs or rows
    uint64_t g = units < 148ull * per_sm ? units : 148ull * per_sm;
    if (g < 1) g = 1;
    kern<<<(unsigned)g, small ? 256 : 512, smem, s>>>(d_in, ld_in, B, L, P, Q,
                                                      reinterpret_cast<const float4 *>(d_tables),
                                                      reinterpret_cast<uint32_t *>(d_out));
    return cudaGetLastError();
}

bool spectral_pack_supported(uint64_t L) {
    return L % 64 == 0 && L / 64 <= 32ull * SPACK_WARPS;
}

cudaError_t launch_spectral_pack(const uint8_t *d_payload, uint64_t bmb, const uint32_t *d_chunk,
                                 const uint64_t *d_meta, uint64_t B, uint32_t L, uint32_t P,
                                 uint32_t Q, const float *d_tables, half_bits *d_out,
                                 cudaStream_t s) {
    if (!spectral_pack_supported(L)) return cudaErrorInvalidValue;
    // dynamic shared memory: the row and its staged coefficients
    const size_t smem = (size_t)srow_halves(L) * 2 + spack_stage_bytes(L);
    if (smem > 220 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(spectral_pack_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    uint64_t g = B < 148ull * 4 ? B : 148ull * 4;
    if (g < 1) g = 1;
    spectral_pack_kernel<<<(unsigned)g, SPACK_THREADS, smem, s>>>(
        d_payload, bmb, d_chunk, rank_group_offset(B * (uint64_t)L), d_meta, B, L, P, Q,
        reinterpret_cast<const float4 *>(d_tables), reinterpret_cast<uint32_t *>(d_out));
    return cudaGetLastError();
}

cudaError_t launch_pack_tables(uint32_t L, uint32_t P, uint32_t Q, float *d_tables,
                               cudaStream_t s) {
    if ((uint64_t)P * Q != L / 2) return cudaErrorInvalidValue;
    pack_tables_kernel<<<(L / 2 + 255) / 256, 256, 0, s>>>(L, P, Q,
                                                            reinterpret_cast<float4 *>(d_tables));
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
