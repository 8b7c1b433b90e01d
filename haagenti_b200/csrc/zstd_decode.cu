// GPU Zstandard decode: one warp per job (a byte range holding one or more
// concatenated frames), several warps per CTA, persistent over the job list.
// The decoder itself is zstd_core.cuh; this file holds the kernel and its
// launcher.  Each warp owns a workspace in shared memory (FSE / Huffman
// tables, repeat offsets, a batch of decoded sequences) and a literal
// scratch area of 128 KiB in device memory.
#include "common.cuh"
#include "zstd_core.cuh"

namespace hct {
namespace {

constexpr int ZWARPS = 4;  // warps (jobs in flight) per CTA
#ifndef ZSTD_MIN_CTAS
#define ZSTD_MIN_CTAS 2  // resident CTAs per SM the register budget allows
#endif
constexpr uint64_t ZSTD_GRID_CAP = 148ull * ZSTD_MIN_CTAS;

__global__ void __launch_bounds__(ZWARPS * 32, ZSTD_MIN_CTAS) zstd_decode_kernel(
    const uint8_t *__restrict__ src, const hct_b200_zstd_job *__restrict__ jobs, uint32_t n,
    uint8_t *dst, hct_b200_status *__restrict__ status, uint8_t *scratch) {
    extern __shared__ uint8_t zsm[];
    __shared__ uint64_t acc[ZWARPS][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    zs::Workspace *ws = reinterpret_cast<zs::Workspace *>(zsm) + warp;
    const uint64_t gw = (uint64_t)blockIdx.x * ZWARPS + warp;
    const uint64_t nw = (uint64_t)gridDim.x * ZWARPS;
    uint8_t *lit = scratch + gw * zs::LIT_SCRATCH;
    for (uint64_t j = gw; j < n; j += nw) {
        const hct_b200_zstd_job jd = jobs[j];
        const zs::Job job{src + jd.src_off, jd.src_len, dst + jd.dst_off, jd.dst_cap, lit};
        const zs::Result r = zs::decode(ws, job, lane, 32, acc[warp]);
        if (lane == 0) {
            hct_b200_status st;
            st.code = r.code;
            st.reserved = 0;
            st.position = r.pos;
            st.provided = jd.dst_cap;
            st.written = r.written;
            status[j] = st;
        }
        __syncwarp();
    }
}

}  // namespace

size_t zstd_scratch_bytes(uint32_t n) {
    const uint64_t ctas = ((uint64_t)n + ZWARPS - 1) / ZWARPS;
    const uint64_t cap = ZSTD_GRID_CAP;
    return (size_t)((ctas < cap ? (ctas ? ctas : 1) : cap) * ZWARPS * zs::LIT_SCRATCH);
}

cudaError_t launch_zstd_decode(const uint8_t *d_src, const hct_b200_zstd_job *d_jobs, uint32_t n,
                               uint8_t *d_dst, hct_b200_status *d_status, uint8_t *d_scratch,
                               cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const size_t smem = sizeof(zs::Workspace) * ZWARPS;
    cudaError_t e = cudaFuncSetAttribute(zstd_decode_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    // as many CTAs as zstd_scratch_bytes provides scratch for
    const uint64_t ctas = ((uint64_t)n + ZWARPS - 1) / ZWARPS;
    const uint64_t grid = ctas < ZSTD_GRID_CAP ? ctas : ZSTD_GRID_CAP;
    zstd_decode_kernel<<<(unsigned)grid, ZWARPS * 32, smem, s>>>(d_src, d_jobs, n, d_dst, d_status,
                                                                 d_scratch);
    return cudaGetLastError();
}

}  // namespace hct
