// K2: INT4 dequantisation with per-block FP16 scales, and the spectral
// scatter that feeds the IDCT contractions.
//
// Value rule (crates/haagenti/src/testing/quantization.rs:82-131):
//     out[i] = f32(nibble_i - 8) * f32(scale[i / 32])
// with the nibble of element i in byte i/2 (low nibble for even i) of the
// section that follows ceil(n/32) little-endian f16 scales.  The f16 -> f32
// conversion is done on the bits (quantization.rs:166-197), so the f32
// product is the same single rounding the reference performs.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace hct {
namespace {

__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
    uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1fu, frac = h & 0x3ffu, out;
    if (exp == 0) {
        if (frac == 0) {
            out = sign << 31;
        } else {  // subnormal: normalise (quantization.rs:173-188)
            int e = -14;
            uint32_t f = frac;
            while ((f & 0x400u) == 0) { f <<= 1; e -= 1; }
            f &= 0x3ffu;
            out = (sign << 31) | ((uint32_t)((e + 127) & 0xff) << 23) | (f << 13);
        }
    } else if (exp == 31) {
        out = (sign << 31) | (0xffu << 23) | (frac << 13);
    } else {
        out = (sign << 31) | ((exp - 15 + 127) << 23) | (frac << 13);
    }
    return __uint_as_float(out);
}

__device__ __forceinline__ float deq(uint32_t nibble, float scale) {
    return __fmul_rn((float)((int)nibble - 8), scale);
}

__device__ __forceinline__ uint16_t to_f16(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ uint16_t to_bf16(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Reads the aligned 32-bit word that holds bytes [p, p+4) of an arbitrary
// byte address p (two aligned loads + funnel shift when p is unaligned).
__device__ __forceinline__ uint32_t ld_u32_any(const uint8_t *p) {
    const uintptr_t a = (uintptr_t)p;
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
    const unsigned sh = (unsigned)(a & 3u);
    if (sh == 0) return w[0];
    return __funnelshift_r(w[0], w[1], 8u * sh);
}

template <int DT>
__device__ __forceinline__ void store8(void *out, uint64_t e, const float v[8], bool vec) {
    if (DT == HCT_B200_F32) {
        float *o = reinterpret_cast<float *>(out) + e;
        if (vec) {
            reinterpret_cast<float4 *>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
            reinterpret_cast<float4 *>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) o[j] = v[j];
        }
    } else {
        uint16_t h[8];
#pragma unroll
        for (int j = 0; j < 8; j++) h[j] = DT == HCT_B200_F16 ? to_f16(v[j]) : to_bf16(v[j]);
        uint16_t *o = reinterpret_cast<uint16_t *>(out) + e;
        if (vec) {
            uint4 u;
            u.x = h[0] | ((uint32_t)h[1] << 16);
            u.y = h[2] | ((uint32_t)h[3] << 16);
            u.z = h[4] | ((uint32_t)h[5] << 16);
            u.w = h[6] | ((uint32_t)h[7] << 16);
            *reinterpret_cast<uint4 *>(o) = u;
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) o[j] = h[j];
        }
    }
}

// One thread per group of 8 elements (4 nibble bytes, one scale).
template <int DT>
__global__ void __launch_bounds__(256) dequant_int4_kernel(const uint8_t *__restrict__ data,
                                                           uint64_t sb, uint64_t n_written,
                                                           void *__restrict__ out, bool vec_ok) {
    const uint8_t *nib = data + sb;
    const uint64_t full_groups = n_written / 8;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < full_groups;
         g += stride) {
        const uint32_t w = ld_u32_any(nib + 4 * g);
        const uint64_t blk = g >> 2;  // 8*g / 32
        const float scale = f16_bits_to_f32((uint32_t)data[2 * blk] | ((uint32_t)data[2 * blk + 1] << 8));
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; j++) v[j] = deq((w >> (4 * j)) & 0xfu, scale);
        store8<DT>(out, 8 * g, v, vec_ok);
    }
    // ragged tail (< 8 elements), byte-wise
    const uint64_t tail0 = full_groups * 8;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid < n_written - tail0) {
        const uint64_t e = tail0 + gid;
        const uint32_t byte = nib[e >> 1];
        const uint32_t nibble = (e & 1) ? (byte >> 4) & 0xfu : byte & 0xfu;
        const uint64_t blk = e >> 5;
        const float scale = f16_bits_to_f32((uint32_t)data[2 * blk] | ((uint32_t)data[2 * blk + 1] << 8));
        const float v = deq(nibble, scale);
        if (DT == HCT_B200_F32) reinterpret_cast<float *>(out)[e] = v;
        else if (DT == HCT_B200_F16) reinterpret_cast<uint16_t *>(out)[e] = to_f16(v);
        else reinterpret_cast<uint16_t *>(out)[e] = to_bf16(v);
    }
}

// ---------------------------------------------------------------- spectral

// Bits [32*w, 32*w+32) of the bitmap, zero past `total` bits / `bmb` bytes.
__device__ __forceinline__ uint32_t bitmap_word(const uint8_t *bm, uint64_t bmb, uint64_t total,
                                                uint64_t w) {
    const uint64_t b0 = 4 * w;
    uint32_t v;
    if (b0 + 4 <= bmb) {
        v = reinterpret_cast<const uint32_t *>(bm)[w];
    } else {
        v = 0;
        for (uint64_t j = 0; j < 4 && b0 + j < bmb; j++) v |= (uint32_t)bm[b0 + j] << (8 * j);
    }
    const uint64_t bit0 = 32 * w;
    if (bit0 >= total) return 0;
    if (total - bit0 < 32) v &= (1u << (uint32_t)(total - bit0)) - 1u;
    return v;
}

// Rank directory, level 1: one CTA per group of RANK_GROUP chunks, one
// thread per 1024-bit chunk (eight 16-byte loads), a block scan of the
// popcounts; writes each chunk's prefix within its group and the group total.
constexpr int RANK_THREADS = (int)RANK_GROUP;

__global__ void __launch_bounds__(RANK_THREADS) chunk_rank_kernel(
    const uint8_t *__restrict__ bm, uint64_t bmb, uint64_t total, uint64_t nchunks,
    uint32_t *__restrict__ local, uint32_t *__restrict__ group_tot) {
    __shared__ uint32_t warp_tot[RANK_THREADS / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t c = (uint64_t)blockIdx.x * RANK_THREADS + threadIdx.x;
    uint32_t cnt = 0;
    if (c < nchunks) {
        if (128 * (c + 1) <= bmb && 1024 * (c + 1) <= total) {
            const uint4 *p = reinterpret_cast<const uint4 *>(bm + 128 * c);
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; j++) v[j] = __ldg(p + j);
#pragma unroll
            for (int j = 0; j < 8; j++)
                cnt += __popc(v[j].x) + __popc(v[j].y) + __popc(v[j].z) + __popc(v[j].w);
        } else {
            for (int j = 0; j < 32; j++) cnt += __popc(bitmap_word(bm, bmb, total, 32 * c + j));
        }
    }
    uint32_t incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    uint32_t before = 0, sum = 0;
#pragma unroll
    for (int w = 0; w < RANK_THREADS / 32; w++) {
        const uint32_t t = warp_tot[w];
        before += w < warp ? t : 0u;
        sum += t;
    }
    if (c < nchunks) local[c] = before + incl - cnt;
    if (threadIdx.x == 0) group_tot[blockIdx.x] = sum;
}

// Exclusive scan of the group totals in place (single CTA of 1024 threads);
// meta[0] = total popcount k, meta[1] = nibble section offset, meta[2] =
// 1 if the payload is too short for k coefficients.
__global__ void __launch_bounds__(1024) chunk_scan_kernel(uint32_t *__restrict__ counts,
                                                          uint64_t nchunks, uint64_t bmb,
                                                          uint64_t payload_len,
                                                          uint64_t *__restrict__ meta,
                                                          int *__restrict__ flag) {
    __shared__ uint32_t warp_sums[32];
    __shared__ uint64_t carry_s;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    if (tid == 0) carry_s = 0;
    __syncthreads();
    for (uint64_t base = 0; base < nchunks; base += 4096) {
        uint32_t v[4];
        uint32_t local = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint64_t i = base + 4 * (uint64_t)tid + j;
            v[j] = i < nchunks ? counts[i] : 0u;
            local += v[j];
        }
        uint32_t incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) warp_sums[wid] = incl;
        __syncthreads();
        if (wid == 0) {
            uint32_t s = warp_sums[lane];
            uint32_t si = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t t = __shfl_up_sync(0xffffffffu, si, o);
                if (lane >= o) si += t;
            }
            warp_sums[lane] = si - s;  // exclusive
        }
        __syncthreads();
        const uint64_t carry = carry_s;
        uint64_t run = carry + warp_sums[wid] + (incl - local);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint64_t i = base + 4 * (uint64_t)tid + j;
            if (i < nchunks) counts[i] = (uint32_t)run;
            run += v[j];
        }
        __syncthreads();
        if (tid == 1023) carry_s = run;
        __syncthreads();
    }
    if (tid == 0) {
        const uint64_t k = carry_s;
        const uint64_t nib_off = bmb + 2 * ((k + 31) / 32);
        meta[0] = k;
        meta[1] = nib_off;
        const bool short_payload = payload_len < nib_off + (k + 1) / 2;
        meta[2] = short_payload ? 1 : 0;
        if (short_payload) atomicExch(flag, HCT_B200_ERR_SIZE_MISMATCH);
    }
}

// One warp per 1024-bit chunk; lane l owns 8 consecutive elements in each of
// 4 passes, so a warp writes 256 contiguous fp16 per pass.
__global__ void __launch_bounds__(256) spectral_scatter_kernel(
    const uint8_t *__restrict__ payload, uint64_t bmb, uint64_t total, uint64_t cols,
    uint64_t nchunks, const uint32_t *__restrict__ chunk_base,
    const uint32_t *__restrict__ group_base, const uint64_t *__restrict__ meta,
    uint16_t *__restrict__ dense, uint64_t ld, bool vec_rows) {
    const int lane = threadIdx.x & 31;
    const uint64_t k = meta[0];
    const uint8_t *scales = payload + bmb;
    const uint8_t *nib = payload + meta[1];
    const bool bad = meta[2] != 0;
    const uint64_t warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t c = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunks;
         c += warps) {
        const uint32_t word = bitmap_word(payload, bmb, total, 32 * c + lane);
        const uint32_t pc = __popc(word);
        uint32_t incl = pc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const uint64_t wrank =
            (uint64_t)chunk_base[c] + group_base[c / RANK_GROUP] + (incl - pc);
#pragma unroll
        for (int pass = 0; pass < 4; pass++) {
            const int src_lane = pass * 8 + (lane >> 2);      // word holding my 8 bits
            const uint32_t wv = __shfl_sync(0xffffffffu, word, src_lane);
            const uint64_t wr = __shfl_sync(0xffffffffu, wrank, src_lane);
            const uint32_t shift = (lane & 3) * 8;
            const uint32_t bits = (wv >> shift) & 0xffu;
            uint64_t r = wr + __popc(wv & ((1u << shift) - 1u));
            const uint64_t e0 = 1024 * c + 256 * pass + 8 * lane;
            uint16_t h[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float v = 0.0f;
                if ((bits >> j) & 1u) {
                    if (!bad && r < k) {
                        const uint32_t byte = nib[r >> 1];
                        const uint32_t nibble = (r & 1) ? (byte >> 4) & 0xfu : byte & 0xfu;
                        const uint64_t sblk = r >> 5;
                        const float scale = f16_bits_to_f32((uint32_t)scales[2 * sblk] |
                                                            ((uint32_t)scales[2 * sblk + 1] << 8));
                        v = deq(nibble, scale);
                    }
                    r++;
                }
                h[j] = to_f16(v);
            }
            if (e0 >= total) continue;
            if (vec_rows && e0 + 8 <= total) {
                const uint64_t row = e0 / cols, col = e0 - row * cols;
                uint4 u;
                u.x = h[0] | ((uint32_t)h[1] << 16);
                u.y = h[2] | ((uint32_t)h[3] << 16);
                u.z = h[4] | ((uint32_t)h[5] << 16);
                u.w = h[6] | ((uint32_t)h[7] << 16);
                *reinterpret_cast<uint4 *>(dense + row * ld + col) = u;
            } else {
                for (int j = 0; j < 8 && e0 + j < total; j++) {
                    const uint64_t e = e0 + j, row = e / cols, col = e - row * cols;
                    dense[row * ld + col] = h[j];
                }
            }
        }
    }
}

// V3 fragment scatter (hct_decoder.h:360-371): the fp16 values vals[0, nvals)
// go, in index order, to the set bits of the fragment's bitmap; set bits past
// nvals are left alone.  overwrite: also write zero at the clear bits and
// the set bits past nvals (the first fragment, onto an unwritten matrix);
// else only the set bits below nvals are written (later fragments).  Same
// warp-per-1024-bit-chunk walk as spectral_scatter_kernel; bm and vals are
// 16- and 2-byte aligned.
__global__ void __launch_bounds__(256) v3_scatter_kernel(
    const uint8_t *__restrict__ bm, uint64_t bmb, uint64_t total, uint64_t cols, uint64_t nchunks,
    const uint32_t *__restrict__ chunk_base, const uint32_t *__restrict__ group_base,
    const uint16_t *__restrict__ vals, uint64_t nvals, uint16_t *__restrict__ dense, uint64_t ld,
    bool vec_rows, bool overwrite) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
    for (uint64_t c = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < nchunks;
         c += warps) {
        const uint32_t word = bitmap_word(bm, bmb, total, 32 * c + lane);
        const uint32_t pc = __popc(word);
        uint32_t incl = pc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const uint64_t wrank =
            (uint64_t)chunk_base[c] + group_base[c / RANK_GROUP] + (incl - pc);
#pragma unroll
        for (int pass = 0; pass < 4; pass++) {
            const int src_lane = pass * 8 + (lane >> 2);  // word holding my 8 bits
            const uint32_t wv = __shfl_sync(0xffffffffu, word, src_lane);
            const uint64_t wr = __shfl_sync(0xffffffffu, wrank, src_lane);
            const uint32_t shift = (lane & 3) * 8;
            const uint32_t bits = (wv >> shift) & 0xffu;
            uint64_t r = wr + __popc(wv & ((1u << shift) - 1u));
            const uint64_t e0 = 1024 * c + 256 * pass + 8 * lane;
            if (e0 >= total) continue;
            uint16_t h[8];
            uint32_t set = 0;  // elements this fragment writes
#pragma unroll
            for (int j = 0; j < 8; j++) {
                h[j] = 0;
                if ((bits >> j) & 1u) {
                    if (r < nvals) {
                        h[j] = vals[r];
                        set |= 1u << j;
                    }
                    r++;
                }
            }
            if (overwrite) set = 0xffu;
            if (!set) continue;
            if (set == 0xffu && vec_rows && e0 + 8 <= total) {
                const uint64_t row = e0 / cols, col = e0 - row * cols;
                uint4 u;
                u.x = h[0] | ((uint32_t)h[1] << 16);
                u.y = h[2] | ((uint32_t)h[3] << 16);
                u.z = h[4] | ((uint32_t)h[5] << 16);
                u.w = h[6] | ((uint32_t)h[7] << 16);
                *reinterpret_cast<uint4 *>(dense + row * ld + col) = u;
            } else {
                for (int j = 0; j < 8 && e0 + j < total; j++) {
                    if (!((set >> j) & 1u)) continue;
                    const uint64_t e = e0 + j, row = e / cols, col = e - row * cols;
                    dense[row * ld + col] = h[j];
                }
            }
        }
    }
}

__global__ void f32_to_f16_padded_kernel(const float *__restrict__ in, uint64_t rows,
                                         uint64_t cols, uint16_t *__restrict__ out, uint64_t ld) {
    const uint64_t n = rows * ld;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t r = i / ld, c = i - r * ld;
        out[i] = c < cols ? to_f16(in[r * cols + c]) : (uint16_t)0;
    }
}

inline unsigned grid_for(uint64_t work, unsigned threads, unsigned max_ctas = 148u * 32u) {
    uint64_t g = (work + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > max_ctas) g = max_ctas;
    return (unsigned)g;
}

}  // namespace

cudaError_t launch_dequant_int4(const uint8_t *d_data, size_t data_len, size_t n_written,
                                size_t num_elements, void *d_out, int dtype, cudaStream_t s) {
    (void)data_len;
    if (n_written == 0) return cudaSuccess;
    const uint64_t nb = (num_elements + 31) / 32;
    const uint64_t sb = nb * 2;
    const bool vec = ((uintptr_t)d_out & 15u) == 0;
    const uint64_t groups = n_written / 8 > 0 ? n_written / 8 : 1;
    const unsigned g = grid_for(groups, 256);
    switch (dtype) {
        case HCT_B200_F32:
            dequant_int4_kernel<HCT_B200_F32><<<g, 256, 0, s>>>(d_data, sb, n_written, d_out, vec);
            break;
        case HCT_B200_F16:
            dequant_int4_kernel<HCT_B200_F16><<<g, 256, 0, s>>>(d_data, sb, n_written, d_out, vec);
            break;
        default:
            dequant_int4_kernel<HCT_B200_BF16><<<g, 256, 0, s>>>(d_data, sb, n_written, d_out, vec);
            break;
    }
    return cudaGetLastError();
}

cudaError_t launch_spectral_scatter(const uint8_t *d_payload, size_t payload_len, uint64_t rows,
                                    uint64_t cols, uint32_t *d_chunk, uint64_t *d_meta,
                                    half_bits *d_dense, uint64_t ld, int *d_flag, cudaStream_t s) {
    const uint64_t total = rows * cols;
    const uint64_t bmb = (total + 7) / 8;
    const uint64_t nchunks = spectral_chunks(total);
    if (ld != cols) {
        cudaError_t e = cudaMemset2DAsync(d_dense + cols, ld * 2, 0, (ld - cols) * 2, rows, s);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = launch_spectral_rank(d_payload, payload_len, total, d_chunk, d_meta, d_flag, s);
    if (e != cudaSuccess) return e;
    const bool vec_rows = (cols % 8 == 0) && (ld % 8 == 0) && (((uintptr_t)d_dense & 15u) == 0);
    spectral_scatter_kernel<<<grid_for(nchunks * 32, 256), 256, 0, s>>>(
        d_payload, bmb, total, cols, nchunks, d_chunk, d_chunk + rank_group_offset(total), d_meta,
        d_dense, ld, vec_rows);
    return cudaGetLastError();
}

cudaError_t launch_v3_scatter(const uint8_t *d_bitmap, uint64_t total, uint64_t cols,
                              const uint16_t *d_vals, uint64_t nvals, uint32_t *d_chunk,
                              uint64_t *d_meta, int *d_flag, half_bits *d_dense, uint64_t ld,
                              bool first, cudaStream_t s) {
    const uint64_t bmb = (total + 7) / 8;
    const uint64_t nchunks = spectral_chunks(total);
    if (first && ld != cols) {  // pad columns zero
        cudaError_t e = cudaMemset2DAsync(d_dense + cols, ld * 2, 0, (ld - cols) * 2,
                                          (total + cols - 1) / cols, s);
        if (e != cudaSuccess) return e;
    }
    // the rank directory only (no INT4 section follows: no short-payload check)
    cudaError_t e = launch_spectral_rank(d_bitmap, ~(size_t)0 >> 2, total, d_chunk, d_meta,
                                         d_flag, s);
    if (e != cudaSuccess) return e;
    const bool vec_rows = (cols % 8 == 0) && (ld % 8 == 0) && (((uintptr_t)d_dense & 15u) == 0);
    v3_scatter_kernel<<<grid_for(nchunks * 32, 256), 256, 0, s>>>(
        d_bitmap, bmb, total, cols, nchunks, d_chunk, d_chunk + rank_group_offset(total), d_vals,
        nvals, d_dense, ld, vec_rows, first);
    return cudaGetLastError();
}

cudaError_t launch_spectral_rank(const uint8_t *d_payload, size_t payload_len, uint64_t total,
                                 uint32_t *d_chunk, uint64_t *d_meta, int *d_flag, cudaStream_t s) {
    const uint64_t bmb = (total + 7) / 8;
    const uint64_t nchunks = spectral_chunks(total);
    const uint64_t groups = (nchunks + RANK_GROUP - 1) / RANK_GROUP;
    uint32_t *group = d_chunk + rank_group_offset(total);
    chunk_rank_kernel<<<(unsigned)(groups ? groups : 1), RANK_THREADS, 0, s>>>(
        d_payload, bmb, total, nchunks, d_chunk, group);
    chunk_scan_kernel<<<1, 1024, 0, s>>>(group, groups, bmb, payload_len, d_meta, d_flag);
    return cudaGetLastError();
}

cudaError_t launch_f32_to_f16_padded(const float *d_in, uint64_t rows, uint64_t cols,
                                     half_bits *d_out, uint64_t ld, cudaStream_t s) {
    f32_to_f16_padded_kernel<<<grid_for(rows * ld, 256), 256, 0, s>>>(d_in, rows, cols, d_out, ld);
    return cudaGetLastError();
}

}  // namespace hct
