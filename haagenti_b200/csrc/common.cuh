// Shared definitions for the hct_b200 kernels and host code.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/hct_b200.h"

namespace hct {

// fp16 buffers are passed as raw 16-bit words.
using half_bits = uint16_t;

// ---- LZ4 (lz4_decode.cu) -----------------------------------------------
cudaError_t launch_lz4_blocks(const uint8_t *d_src, const hct_b200_lz4_block *d_blocks,
                              uint32_t n, uint8_t *d_dst, hct_b200_status *d_status,
                              cudaStream_t s);

// ---- INT4 / spectral scatter (int4_dequant.cu) -------------------------
// n_written elements are produced (the reference's short-input rule is
// applied by the caller), out_dtype one of HCT_B200_F32/F16/BF16.
cudaError_t launch_dequant_int4(const uint8_t *d_data, size_t data_len, size_t n_written,
                                size_t num_elements, void *d_out, int out_dtype, cudaStream_t s);

// Number of 1024-bit chunks the spectral scatter scans.
inline uint64_t spectral_chunks(uint64_t total) { return (total + 1023) / 1024; }

// Spectral payload (bitmap ++ INT4) -> dense fp16 coefficients, row stride ld
// (ld >= cols, pad columns written as zero).  Scratch: d_chunk holds
// spectral_chunks(total)+1 u32, d_meta 4 u64 (meta[0] = popcount k).
cudaError_t launch_spectral_scatter(const uint8_t *d_payload, size_t payload_len, uint64_t rows,
                                    uint64_t cols, uint32_t *d_chunk, uint64_t *d_meta,
                                    half_bits *d_dense, uint64_t ld, int *d_flag, cudaStream_t s);

// f32 row-major rows x cols -> fp16 with row stride ld (zero padded).
cudaError_t launch_f32_to_f16_padded(const float *d_in, uint64_t rows, uint64_t cols,
                                     half_bits *d_out, uint64_t ld, cudaStream_t s);

// ---- DCT basis + tcgen05 contraction (idct_gemm.cu) -------------------
// basis[i][k] = alpha(k) cos(pi (2i+1) k / 2n), fp16, row stride ld (zero padded).
cudaError_t launch_basis(const double *d_cos_table, uint64_t n, half_bits *d_basis, uint64_t ld,
                         cudaStream_t s);

// C[M x N] = A[M x K] . B[N x K]^T, A/B fp16 K-major with row strides lda/ldb
// (multiples of 8 elements).  Epilogue:
//   mode 0: C^T stored fp16 at out[n * ldo + m]          (transposed)
//   mode 1: C stored out_dtype at out[m * ldo + n]         (row-major)
struct GemmArgs {
    const half_bits *A;
    const half_bits *B;
    uint64_t M, N, K;
    uint64_t lda, ldb;
    void *out;
    uint64_t ldo;
    int mode;
    int out_dtype;
    int *d_flag;  // device error flag (HCT_B200_ERR_TIMEOUT on an expired wait)
};
cudaError_t launch_umma_gemm(const GemmArgs &args, cudaStream_t s);

}  // namespace hct
