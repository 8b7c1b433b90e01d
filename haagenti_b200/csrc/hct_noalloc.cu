// Allocation-free spectral decode for small tensors.
//
// Some callers cannot allocate device memory when they decode: a runtime
// whose allocator has already carved out (or is sizing) the whole of HBM for
// its own pools, an allocator-owning host process that forbids stray
// cudaMalloc/cudaFree (which synchronise the device and fragment its pool),
// or code running where creating a context with its own scratch is not
// possible.  For them this file offers one entry point that performs the
// same work as hct_b200_spectral_q4_decode (INT4 dequantisation + bitmap
// scatter + the two tcgen05 IDCT contractions) but takes all of its scratch
// from a fixed, file-scope device array instead of a context.
//
// The array is 32 MiB plus a few KiB, so the entry point serves tensors of at
// most NOALLOC_MAX_DIM rows and columns (rows * cols <= NOALLOC_MAX_ELEMS);
// larger requests are rejected with HCT_B200_ERR_INVALID_ARGUMENT before any
// GPU work.  Every process that loads the library holds this array on each
// device it touches, until it exits.
//
// All calls share the one array: two calls whose GPU work overlaps (other
// streams, other host threads) race on it and must be serialised by the
// caller.  The array keeps the last call's contents; each call rewrites
// everything it reads back (the error flag is cleared, the bases and the
// coefficient matrices are regenerated).
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"

namespace {

constexpr uint64_t NOALLOC_MAX_DIM = 2048;
constexpr uint64_t NOALLOC_MAX_ELEMS = NOALLOC_MAX_DIM * NOALLOC_MAX_DIM;

// Byte offsets inside the scratch array (each region 256-byte aligned).
constexpr size_t OFF_FLAG = 0;
constexpr size_t OFF_META = 256;
constexpr size_t OFF_CHUNK = 512;
constexpr size_t CHUNK_BYTES = (hct::rank_dir_words(NOALLOC_MAX_ELEMS) * 4 + 255) / 256 * 256;
constexpr size_t MAT_BYTES = NOALLOC_MAX_ELEMS * 2;  // one fp16 matrix, <= 2048 x 2048
constexpr size_t OFF_BASIS_W = OFF_CHUNK + CHUNK_BYTES;
constexpr size_t OFF_BASIS_H = OFF_BASIS_W + MAT_BYTES;
constexpr size_t OFF_DENSE = OFF_BASIS_H + MAT_BYTES;
constexpr size_t OFF_TT = OFF_DENSE + MAT_BYTES;
constexpr size_t SCRATCH_BYTES = OFF_TT + MAT_BYTES;  // 33,571,328 bytes

// The scratch itself.  In host code `g_noalloc_scratch` names a host-side
// stand-in, not device memory: its device address comes from
// cudaGetSymbolAddress, looked up once per device below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_lookup_mu;
uint8_t *g_scratch_ptr[MAX_DEVICES] = {};

// Device address of the scratch array on the current device (set-up on the
// first call made on each device).
int scratch_on_current_device(uint8_t **out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES)
        return HCT_B200_ERR_NO_DEVICE;
    std::lock_guard<std::mutex> g(g_lookup_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return HCT_B200_ERR_CUDA;
        g_scratch_ptr[dev] = static_cast<uint8_t *>(p);
    }
    *out = g_scratch_ptr[dev];
    return HCT_B200_OK;
}

// DCT-III basis b[i][k] = alpha(k) cos(pi (2i+1) k / 2n) in fp16, row stride
// ld; the angle is reduced exactly in integers before cospi().
__global__ void noalloc_basis_kernel(uint64_t n, uint16_t *__restrict__ out, uint64_t ld) {
    const uint64_t total = n * ld;
    const double a0 = sqrt(1.0 / (double)n), a1 = sqrt(2.0 / (double)n);
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t i = idx / ld, k = idx - i * ld;
        uint16_t h = 0;
        if (k < n) {
            const uint64_t j = ((2 * i + 1) * k) % (4 * n);
            h = __half_as_ushort(__double2half((k == 0 ? a0 : a1) * cospi((double)j / (2.0 * n))));
        }
        out[idx] = h;
    }
}

inline uint64_t round8(uint64_t v) { return (v + 7) / 8 * 8; }

int launch_basis_noalloc(uint64_t n, uint16_t *dst, cudaStream_t s) {
    const uint64_t total = n * round8(n);
    uint64_t g = (total + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    noalloc_basis_kernel<<<(unsigned)g, 256, 0, s>>>(n, dst, round8(n));
    return cudaGetLastError() == cudaSuccess ? HCT_B200_OK : HCT_B200_ERR_CUDA;
}

}  // namespace

extern "C" int hct_b200_spectral_q4_decode_noalloc(const uint8_t *d_payload, size_t payload_len,
                                                   size_t rows_in, size_t cols_in, void *d_out,
                                                   int out_dtype, void *stream) {
    using namespace hct;
    if (!d_payload || !d_out) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)d_payload & 15u) != 0) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (rows_in == 0 || cols_in == 0) return HCT_B200_OK;
    if (rows_in > NOALLOC_MAX_DIM || cols_in > NOALLOC_MAX_DIM) return HCT_B200_ERR_INVALID_ARGUMENT;
    uint64_t rows = rows_in, cols = cols_in;
    if (cols == 1 && rows > 1) {  // a column vector is one row transform
        rows = 1;
        cols = rows_in;
    }
    const uint64_t total = rows * cols;
    if (payload_len < (total + 7) / 8) return HCT_B200_ERR_SIZE_MISMATCH;

    uint8_t *base = nullptr;
    int rc = scratch_on_current_device(&base);
    if (rc) return rc;
    cudaStream_t s = (cudaStream_t)stream;
    int *flag = reinterpret_cast<int *>(base + OFF_FLAG);
    uint64_t *meta = reinterpret_cast<uint64_t *>(base + OFF_META);
    uint32_t *chunk = reinterpret_cast<uint32_t *>(base + OFF_CHUNK);
    half_bits *basis_w = reinterpret_cast<half_bits *>(base + OFF_BASIS_W);
    half_bits *basis_h = reinterpret_cast<half_bits *>(base + OFF_BASIS_H);
    half_bits *dense = reinterpret_cast<half_bits *>(base + OFF_DENSE);
    half_bits *tt = reinterpret_cast<half_bits *>(base + OFF_TT);
    const uint64_t ldw = round8(cols), ldh = round8(rows);

    if (cudaMemsetAsync(flag, 0, sizeof(int), s) != cudaSuccess) return HCT_B200_ERR_CUDA;
    if (launch_spectral_scatter(d_payload, payload_len, rows, cols, chunk, meta, dense, ldw, flag, s) !=
        cudaSuccess)
        return HCT_B200_ERR_CUDA;
    rc = launch_basis_noalloc(cols, basis_w, s);
    if (rc) return rc;
    if (rows == 1) {
        GemmArgs g{dense, basis_w, rows, cols, cols, ldw, ldw, d_out, cols, 1, out_dtype, flag};
        if (launch_umma_gemm(g, s) != cudaSuccess) return HCT_B200_ERR_CUDA;
    } else {
        rc = launch_basis_noalloc(rows, basis_h, s);
        if (rc) return rc;
        GemmArgs g1{dense, basis_w, rows, cols, cols, ldw, ldw, tt, ldh, 0, HCT_B200_F16, flag};
        if (launch_umma_gemm(g1, s) != cudaSuccess) return HCT_B200_ERR_CUDA;
        GemmArgs g2{basis_h, tt, rows, cols, rows, ldh, ldh, d_out, cols, 1, out_dtype, flag};
        if (launch_umma_gemm(g2, s) != cudaSuccess) return HCT_B200_ERR_CUDA;
    }
    int f = 0;
    if (cudaMemcpyAsync(&f, flag, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return HCT_B200_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return HCT_B200_ERR_CUDA;
    return f;
}
