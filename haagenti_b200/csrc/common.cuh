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
// max_src_len: an upper bound of the blocks' compressed lengths when the
// caller knows one (0 = unknown); bounds up to the LZ4 bound of a 16 KiB
// block select the variant that stages each compressed block in shared memory.
cudaError_t launch_lz4_blocks(const uint8_t *d_src, const hct_b200_lz4_block *d_blocks,
                              uint32_t n, uint8_t *d_dst, hct_b200_status *d_status,
                              cudaStream_t s, uint64_t max_src_len = 0);

// ---- INT4 / spectral scatter (int4_dequant.cu) -------------------------
// n_written elements are produced (the reference's short-input rule is
// applied by the caller), out_dtype one of HCT_B200_F32/F16/BF16.  d_flag
// receives HCT_B200_ERR_TIMEOUT if a bounded wait on a staged copy expires.
cudaError_t launch_dequant_int4(const uint8_t *d_data, size_t data_len, size_t n_written,
                                size_t num_elements, void *d_out, int out_dtype, int *d_flag,
                                cudaStream_t s);
// Many tensors in few launches (DQ_MAX_JOBS per launch).
struct Int4Job {
    const uint8_t *data;   // scales then nibbles (the quantize_int4 layout)
    void *out;
    uint64_t num_elements; // sets the scale section: 2 * ceil(num_elements / 32) bytes
    uint64_t n_written;    // elements to produce (<= num_elements)
};
constexpr uint32_t DQ_MAX_JOBS = 64;
cudaError_t launch_dequant_int4_batch(const Int4Job *jobs, uint32_t njobs, int out_dtype,
                                      int *d_flag, cudaStream_t s);

// Number of 1024-bit chunks the spectral scatter scans.
__host__ __device__ inline constexpr uint64_t spectral_chunks(uint64_t total) {
    return (total + 1023) / 1024;
}
// Rank directory of the bitmap (launch_spectral_rank): d_chunk[c] is the
// popcount of the chunks before c within its group of RANK_GROUP chunks, and
// the group prefixes follow at d_chunk + rank_group_offset(total), so the
// rank of chunk c is d_chunk[c] + d_chunk[rank_group_offset + c / RANK_GROUP].
constexpr uint64_t RANK_GROUP = 256;
__host__ __device__ inline constexpr uint64_t rank_group_offset(uint64_t total) {
    return (spectral_chunks(total) + RANK_GROUP - 1) / RANK_GROUP * RANK_GROUP;
}
// u32 words of the rank directory for a bitmap of `total` bits.
__host__ __device__ inline constexpr uint64_t rank_dir_words(uint64_t total) {
    return rank_group_offset(total) + spectral_chunks(total) / RANK_GROUP + 2;
}

// Spectral payload (bitmap ++ INT4) -> dense fp16 coefficients, row stride ld
// (ld >= cols, pad columns written as zero).  Scratch: d_chunk holds
// rank_dir_words(total) u32, d_meta 4 u64 (meta[0] = popcount k).
cudaError_t launch_spectral_scatter(const uint8_t *d_payload, size_t payload_len, uint64_t rows,
                                    uint64_t cols, uint32_t *d_chunk, uint64_t *d_meta,
                                    half_bits *d_dense, uint64_t ld, int *d_flag, cudaStream_t s);

// One V3 fragment (bitmap ++ fp16 values) scattered into the dense fp16
// matrix: its values at its set bits in index order (set bits past nvals
// keep their value).  first: the matrix is unwritten, so clear bits (and pad
// columns) are written as zero.  d_bitmap 16-byte and d_vals 2-byte aligned.
cudaError_t launch_v3_scatter(const uint8_t *d_bitmap, uint64_t total, uint64_t cols,
                              const uint16_t *d_vals, uint64_t nvals, uint32_t *d_chunk,
                              uint64_t *d_meta, int *d_flag, half_bits *d_dense, uint64_t ld,
                              bool first, cudaStream_t s);

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
//   mode 2: DFT stage 1 of the factored IDCT (fdct.cu): row R = (b, k2), the
//           complex output m1 = column pair (2m1, 2m1+1), times twiddle[k2*m1],
//           stored as fp16 pair at ((m1 * batch + b) * Q + k2); N = 2P (<= 256
//           on the persistent stage kernel, any even N on the tiled one)
//   mode 3: DFT stage 2: row R = (m1, b), complex output m2, j = m1 + P*m2,
//           scaled and scattered to out[(4j + 2 ri) * ldo + b] (j < H/2) or
//           out[(4(H-1-j) + 3 - 2 ri) * ldo + b] in out_dtype
//   mode 4: DFT stage 1 with the twiddle folded into per-k2 matrices: A holds
//           Z as [k2][b][k1] (rows (k2, b), batch % 128 == 0), B is a table of
//           Q matrices of stage_w_rows(N, K) rows each (N = 2P live rows);
//           output G[m1][k2][ri][b] fp16
//   mode 5: DFT stage 2 reading that G as an MN-major operand (A = G, lda =
//           batch, K = 2Q a multiple of 64); output as mode 3
//   mode 6: DFT stage 1 with the Makhoul pack and the twiddle folded into
//           per-pair matrices: A holds the lines x as T'[n][k2][r] = x[Q r + k2]
//           (batch lines of stride lda, 64 <= 2P <= 128, P % 4 == 0), a tile
//           reads columns u and (Q - u) mod Q of 128 lines, B is the table of
//           launch_makhoul_fold_table (N = 256 rows per pair, K = 128 kbc),
//           M = (Q/2 + 1) batch; output G[m1][k2][ri][b] fp16 as mode 4
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
    // factored-DCT stage parameters (modes 2 and 3)
    uint32_t P = 0, Q = 0, H = 0;
    uint64_t batch = 0;
    const float *twiddle = nullptr;  // e^{2 pi i j / H}, complex fp32 (mode 2)
    float scale = 1.0f;              // mode 3
    // modes 2 and 3: a device word for dynamic tile scheduling (CTAs take the
    // next tile from it, so CTAs that start late do fewer tiles); cleared by
    // the launch.  nullptr: tiles are dealt out statically.
    uint32_t *tile_counter = nullptr;
};
cudaError_t launch_umma_gemm(const GemmArgs &args, cudaStream_t s);
// rows of each per-k2 matrix of mode 4 (the stage kernel's resident W height)
uint32_t stage_w_rows(uint64_t N, uint64_t K);
// The mode-4 table: for k2 < Q, rows o = 2 m1 + ri (< 2P; zero up to w_rows)
// and columns k = 2 k1 + rk (< 2P; zero up to ld), the realified
// e^{2 pi i m1 (Q k1 + k2) / H}.
cudaError_t launch_twiddled_dft_table(uint32_t P, uint32_t Q, uint32_t w_rows, uint32_t ld,
                                      half_bits *d_out, cudaStream_t s);
// The mode-6 table: for each pair u in [0, Q/2], 256 rows (G of k2 = u, then
// of k2 = Q - u) x 128 kbc columns (kbc = ceil(2P / 64) values of column u,
// then of column (Q - u) mod Q), fp16; (Q/2 + 1) 256 128 kbc entries.
cudaError_t launch_makhoul_fold_table(uint32_t P, uint32_t Q, uint32_t kbc, half_bits *d_out,
                                      cudaStream_t s);

// ---- factored DCT-III (fdct.cu) -----------------------------------------
// L even, H = L/2 = P*Q: preferably P, Q multiples of 4 and <= 128 (the most
// balanced such split); otherwise Q the largest multiple of 4 <= 128 dividing
// H and P = H/Q <= FDCT_MAX_P of any residue (the vocabulary lengths).
constexpr uint32_t FDCT_MAX_P = 4096;
bool fdct_factor(uint64_t L, uint32_t *P, uint32_t *Q);
// complex values per (b, k2) row of the pack's output Z: P, or P rounded up
// to a multiple of 8 (zero padded) when P is not a multiple of 4
uint32_t fdct_padded_p(uint32_t P);
// rows of length L (fp16, stride ld_in) -> Z[b][k2][k1] complex fp16 pairs,
// rows of fdct_padded_p(P) values.  d_tables: the per-k pack coefficients
// (natural k order) written by launch_pack_tables(L, P, Q).
// k2_major: Z laid out [k2][b][k1] instead (the input of DFT stage mode 4).
// perm_q != 0: line b is written at slot (b % perm_q) perm_2p + b / perm_q
// (perm_q perm_2p == batch), the order whose transposed result the next
// pass reads with stage mode 6 (Q = perm_q, 2P = perm_2p of that pass).
cudaError_t launch_makhoul_pack(const half_bits *d_in, uint64_t ld_in, uint64_t batch, uint32_t L,
                                uint32_t P, uint32_t Q, const float *d_tables, half_bits *d_out,
                                bool k2_major, uint32_t perm_q, uint32_t perm_2p, cudaStream_t s);
// L/2 float4 (alpha_k, beta_k) in natural k order (P Q = L/2).
cudaError_t launch_pack_tables(uint32_t L, uint32_t P, uint32_t Q, float *d_tables,
                               cudaStream_t s);
// Rank directory of a spectral payload (layout at spectral_chunks above) in
// d_chunk, meta[0] = k, meta[1] = nibble offset, meta[2] = short.
cudaError_t launch_spectral_rank(const uint8_t *d_payload, size_t payload_len, uint64_t total,
                                 uint32_t *d_chunk, uint64_t *d_meta, int *d_flag, cudaStream_t s);
// Row pack straight from a spectral payload (rows of length L, row-major
// bitmap), after launch_spectral_rank.  Needs spectral_pack_supported(L).
bool spectral_pack_supported(uint64_t L);
cudaError_t launch_spectral_pack(const uint8_t *d_payload, uint64_t bmb, const uint32_t *d_chunk,
                                 const uint64_t *d_meta, uint64_t batch, uint32_t L, uint32_t P,
                                 uint32_t Q, const float *d_tables, half_bits *d_out,
                                 bool k2_major, uint32_t perm_q, uint32_t perm_2p,
                                 cudaStream_t s, bool transposed = false);
// transposed: no pack; each line is written as out[slot][k2][r] = c[Q r + k2]
// (L values per line), the input of stage mode 6 (Q % 8 == 0, 2P <= 128).
// ---- HoloTensor SV03 fragments (holo.cu) ---------------------------------
// One residue class r of the raster positions p = r + F i: fragment values
// vals[src + i - q0] for q0 <= i < q0 + count, no fragment when count == 0.
struct Sv03Residue {
    uint64_t src, q0, count;
};
// dense[b][k] (fp16, row stride ldw) = value of raster position b cols + k
// from its residue (zero where none), for all rows x cols; F > 0.
cudaError_t launch_sv03_interleave(const float *d_vals, const Sv03Residue *d_res, uint32_t F,
                                   uint64_t rows, uint64_t cols, half_bits *d_dense, uint64_t ldw,
                                   cudaStream_t s);
// One fragment's values at positions start + j F (< n), j < count; F == 0
// writes the last value at start.  The matrix must be cleared beforehand.
cudaError_t launch_sv03_scatter(const float *d_vals, uint64_t count, uint64_t start, uint64_t F,
                                uint64_t n, uint64_t cols, half_bits *d_dense, uint64_t ldw,
                                cudaStream_t s);

// ---- Zstandard (zstd_decode.cu) --------------------------------------------
// Device scratch for launch_zstd_decode over n jobs (128 KiB of literals per
// warp in flight).
size_t zstd_scratch_bytes(uint32_t n);
cudaError_t launch_zstd_decode(const uint8_t *d_src, const hct_b200_zstd_job *d_jobs, uint32_t n,
                               uint8_t *d_dst, hct_b200_status *d_status, uint8_t *d_scratch,
                               cudaStream_t s);

// realified n-point inverse-DFT matrix, 2n x 2n fp16 (rows_pad x ld).
cudaError_t launch_dft_matrix(uint32_t n, uint32_t rows_pad, uint32_t ld, half_bits *d_out,
                              cudaStream_t s);
cudaError_t launch_twiddle_table(uint32_t H, float *d_out, cudaStream_t s);

}  // namespace hct
