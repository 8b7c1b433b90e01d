// HoloTensor spectral fragments ("SV03") into the dense coefficient matrix
// that the IDCT reads.
//
// SpectralEncoder::encode_2d (crates/haagenti-hct/src/holotensor.rs:734-780)
// deals the raster-order f32 DCT coefficients out to F fragments: fragment
// f holds positions start_f, start_f + F, start_f + 2F, ...
// SpectralDecoder::add_fragment_v3 (holotensor.rs:979-1015) writes them
// back into an accumulator, later fragments overwriting earlier ones, and
// reconstruct (holotensor.rs:1029-1051) runs idct_2d on it.
//
// sv03_interleave_kernel covers the usual case (one stride F for every
// loaded fragment, distinct residues start_f mod F): it is output-major, so
// every output row is written once with 16-byte stores and each fragment's
// values are read in order.  Any other set of fragments goes through
// sv03_scatter_kernel, one launch per fragment in load order, which keeps
// the reference's last-writer-wins rule exactly.
#include <cuda_fp16.h>

#include "common.cuh"

namespace hct {
namespace {

__device__ __forceinline__ uint32_t f2h_bits(float v) {
    return (uint32_t)__half_as_ushort(__float2half_rn(v));
}

// dense[b][k] (row stride ldw, fp16) for b < rows, k < cols: raster position
// p = b cols + k has residue r = p mod F and slice index i = p div F; the
// value is vals[res[r].src + i - res[r].q0] when q0 <= i < q0 + count (else
// zero).  Each thread writes 8 consecutive k of one row.
__global__ void __launch_bounds__(256) sv03_interleave_kernel(
    const float *__restrict__ vals, const Sv03Residue *__restrict__ res, uint32_t F,
    uint64_t rows, uint64_t cols, uint16_t *__restrict__ dense, uint64_t ldw) {
    const uint64_t groups = (cols + 7) / 8;
    const uint64_t total = rows * groups;
    const bool vec = (ldw % 8 == 0) && (((uintptr_t)dense & 15) == 0);
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t b = t / groups, k0 = 8 * (t - b * groups);
        const uint64_t p0 = b * cols + k0;
        uint64_t i = p0 / F;
        uint32_t r = (uint32_t)(p0 - i * F);
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t v = 0;
            if (k0 + j < cols) {
                const Sv03Residue e = res[r];
                if (i >= e.q0 && i - e.q0 < e.count) v = f2h_bits(vals[e.src + (i - e.q0)]);
            }
            h[j] = v;
            if (++r == F) {
                r = 0;
                ++i;
            }
        }
        uint16_t *o = dense + b * ldw + k0;
        if (vec && k0 + 8 <= ldw) {
            *reinterpret_cast<uint4 *>(o) = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16),
                                                       h[4] | (h[5] << 16), h[6] | (h[7] << 16));
        } else {
            for (int j = 0; j < 8; j++)
                if (k0 + j < cols) o[j] = (uint16_t)h[j];
        }
    }
}

// One fragment: positions start + j F (j < count, position < n) get
// vals[j]; with F == 0 the single position start gets the last value.
__global__ void __launch_bounds__(256) sv03_scatter_kernel(
    const float *__restrict__ vals, uint64_t count, uint64_t start, uint64_t F, uint64_t n,
    uint64_t cols, uint16_t *__restrict__ dense, uint64_t ldw) {
    for (uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; j < count;
         j += (uint64_t)gridDim.x * blockDim.x) {
        if (F == 0 && j + 1 != count) continue;
        const uint64_t p = start + F * j;
        if (p >= n) continue;
        const uint64_t b = p / cols;
        dense[b * ldw + (p - b * cols)] = (uint16_t)f2h_bits(vals[j]);
    }
}

}  // namespace

cudaError_t launch_sv03_interleave(const float *d_vals, const Sv03Residue *d_res, uint32_t F,
                                   uint64_t rows, uint64_t cols, half_bits *d_dense, uint64_t ldw,
                                   cudaStream_t s) {
    if (F == 0) return cudaErrorInvalidValue;
    const uint64_t total = rows * ((cols + 7) / 8);
    uint64_t g = (total + 255) / 256;
    if (g > 148ull * 16) g = 148ull * 16;
    if (g < 1) g = 1;
    sv03_interleave_kernel<<<(unsigned)g, 256, 0, s>>>(d_vals, d_res, F, rows, cols,
                                                        reinterpret_cast<uint16_t *>(d_dense), ldw);
    return cudaGetLastError();
}

cudaError_t launch_sv03_scatter(const float *d_vals, uint64_t count, uint64_t start, uint64_t F,
                                uint64_t n, uint64_t cols, half_bits *d_dense, uint64_t ldw,
                                cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    uint64_t g = (count + 255) / 256;
    if (g > 148ull * 16) g = 148ull * 16;
    sv03_scatter_kernel<<<(unsigned)g, 256, 0, s>>>(d_vals, count, start, F, n, cols,
                                                     reinterpret_cast<uint16_t *>(d_dense), ldw);
    return cudaGetLastError();
}

}  // namespace hct
