// K3: the inverse DCT as two dense contractions against the DCT basis on
// tcgen05 tensor cores (sm_100a).
//
// The reference's idct_2d (crates/haagenti-core/src/dct.rs:311-337) applies
// the orthonormal DCT-III along columns and then along rows of the
// height x width coefficient matrix F, i.e.
//     X = A_H . F . A_W^T,   A_n[i][k] = alpha(k) cos(pi (2i+1) k / 2n),
//     alpha(0) = sqrt(1/n), alpha(k>0) = sqrt(2/n).
// Here that is two GEMMs with fp16 operands and fp32 accumulation:
//     GEMM 1:  T^T = (F . A_W^T)^T       (A = F,   B = A_W,  K = width)
//     GEMM 2:  X   = A_H . T             (A = A_H, B = T^T,  K = height)
// Both are "C = A . B^T" with K-major operands, so one kernel serves both;
// GEMM 1 writes its tile transposed so GEMM 2's B operand is K-major too.
//
// Kernel structure (one 128 x 256 output tile per CTA, 6 warps):
//   warp 0  TMA producer: 128B-swizzled A/B tiles into a 4-stage ring,
//           completion signalled on the stage's "full" mbarrier;
//   warp 1  TMEM allocator + single-thread tcgen05.mma issuer; each stage
//           is released to the producer by tcgen05.commit on "empty";
//   warps 2-5 epilogue: tcgen05.ld of the fp32 accumulator (TMEM lanes =
//           tile rows), conversion and global stores.
// Every mbarrier wait is bounded (iteration count and %globaltimer); an
// expired wait raises HCT_B200_ERR_TIMEOUT in the device flag, the CTA
// drains its own in-flight copies and MMAs (again bounded), frees TMEM and
// exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"

namespace hct {
namespace {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 fp16 = 128 bytes = one 128B swizzle row
constexpr int STAGES = 4;
constexpr int A_TILE_BYTES = BM * BK * 2;
constexpr int B_TILE_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
constexpr int TMEM_COLS = 256;
constexpr int THREADS = 192;
constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + (size_t)STAGES * STAGE_BYTES + 256;

constexpr uint64_t WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s per wait
constexpr uint32_t WAIT_MAX_ITERS = 1u << 30;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: false when the phase did not complete in time.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t i = 1; i < WAIT_MAX_ITERS; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && globaltimer() - t0 > WAIT_TIMEOUT_NS) return false;
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// UMMA shared-memory descriptor, K-major, 128B swizzle: rows of 128 bytes,
// 8-row core groups 1024 bytes apart (SBO), LBO unused (1), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// Instruction descriptor: kind::f16, A = B = fp16, D = f32, both K-major,
// N = 256 (bits 17..22 hold N>>3), M = 128 (bits 24..28 hold M>>4).
constexpr uint32_t IDESC = (1u << 4) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(IDESC), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct SmemCtl {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t accum;
    uint32_t tmem_base;
    int abort;
    int consumed;  // k-blocks whose "full" phase the MMA thread observed
    int issued;    // k-blocks whose TMA loads were issued
    int mma_issued;
};

__device__ __forceinline__ void raise_timeout(int *flag, SmemCtl *ctl) {
    atomicExch(flag, HCT_B200_ERR_TIMEOUT);
    atomicExch(&ctl->abort, 1);
}

__device__ __forceinline__ uint16_t f2h(float v) { return __half_as_ushort(__float2half_rn(v)); }
__device__ __forceinline__ uint16_t f2bf(float v) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__global__ void __launch_bounds__(THREADS, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, uint32_t M, uint32_t N, uint32_t K,
                     uint32_t m_tiles, void *out, uint64_t ldo, int mode, int out_dtype,
                     int *flag) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    SmemCtl *ctl = reinterpret_cast<SmemCtl *>(smem + (size_t)STAGES * STAGE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t m_tile = blockIdx.x % m_tiles, n_tile = blockIdx.x / m_tiles;
    const int m0 = (int)(m_tile * BM), n0 = (int)(n_tile * BN);
    const int num_kb = (int)((K + BK - 1) / BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(smem_u32(&ctl->full[s]), 1);
            mbar_init(smem_u32(&ctl->empty[s]), 1);
        }
        mbar_init(smem_u32(&ctl->accum), 1);
        ctl->abort = 0;
        ctl->consumed = 0;
        ctl->issued = 0;
        ctl->mma_issued = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA))
                         : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB))
                         : "memory");
            for (int kb = 0; kb < num_kb; kb++) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (*(volatile int *)&ctl->abort) break;
                if (!mbar_wait(smem_u32(&ctl->empty[s]), ph ^ 1u)) {
                    raise_timeout(flag, ctl);
                    break;
                }
                const uint32_t sa = smem_u32(smem + (size_t)s * STAGE_BYTES);
                const uint32_t sb = sa + A_TILE_BYTES;
                const uint32_t fb = smem_u32(&ctl->full[s]);
                mbar_expect_tx(fb, STAGE_BYTES);
                tma_load_2d(sa, &tmA, fb, kb * BK, m0);
                tma_load_2d(sb, &tmB, fb, kb * BK, n0);
                *(volatile int *)&ctl->issued = kb + 1;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            int kb = 0;
            for (; kb < num_kb; kb++) {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
                if (*(volatile int *)&ctl->abort) break;
                if (!mbar_wait(smem_u32(&ctl->full[s]), ph)) {
                    raise_timeout(flag, ctl);
                    break;
                }
                *(volatile int *)&ctl->consumed = kb + 1;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t sa = smem_u32(smem + (size_t)s * STAGE_BYTES);
                const uint32_t sb = sa + A_TILE_BYTES;
                const uint64_t da = umma_desc_sw128(sa), db = umma_desc_sw128(sb);
#pragma unroll
                for (int k = 0; k < BK / 16; k++) {
                    // +32 bytes along K inside the swizzle row = +2 in the address field
                    umma_f16(tmem, da + 2 * k, db + 2 * k, (kb | k) != 0);
                }
                umma_commit(smem_u32(&ctl->empty[s]));
                ctl->mma_issued = 1;
            }
            // Signals the epilogue (and the teardown) once every MMA issued
            // above has completed; also issued on the abort path.
            umma_commit(smem_u32(&ctl->accum));
        }
    } else {
        // epilogue warps 2..5 -> TMEM lane quarter (warp % 4)
        const int q = warp & 3;
        const bool ok = mbar_wait(smem_u32(&ctl->accum), 0);
        if (!ok) raise_timeout(flag, ctl);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok && !*(volatile int *)&ctl->abort) {
            const int row = m0 + q * 32 + lane;
            const bool row_ok = row < (int)M;
            for (int c = 0; c < BN; c += 32) {
                uint32_t r[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
                const int col0 = n0 + c;
                if (!row_ok || col0 >= (int)N) continue;
                const int ncols = min(32, (int)N - col0);
                if (mode == 0) {
                    uint16_t *o = reinterpret_cast<uint16_t *>(out);
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (j < ncols) o[(uint64_t)(col0 + j) * ldo + row] = f2h(__uint_as_float(r[j]));
                } else if (out_dtype == HCT_B200_F32) {
                    float *o = reinterpret_cast<float *>(out) + (uint64_t)row * ldo + col0;
                    if (ncols == 32 && ((uintptr_t)o & 15u) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(o + j) =
                                make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                            __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (j < ncols) o[j] = __uint_as_float(r[j]);
                    }
                } else {
                    uint16_t *o = reinterpret_cast<uint16_t *>(out) + (uint64_t)row * ldo + col0;
                    const bool bf = out_dtype == HCT_B200_BF16;
                    if (ncols == 32 && ((uintptr_t)o & 15u) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint32_t w[4];
#pragma unroll
                            for (int t = 0; t < 4; t++) {
                                const float a = __uint_as_float(r[j + 2 * t]);
                                const float b = __uint_as_float(r[j + 2 * t + 1]);
                                w[t] = bf ? ((uint32_t)f2bf(a) | ((uint32_t)f2bf(b) << 16))
                                          : ((uint32_t)f2h(a) | ((uint32_t)f2h(b) << 16));
                            }
                            *reinterpret_cast<uint4 *>(o + j) = make_uint4(w[0], w[1], w[2], w[3]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            const float a = __uint_as_float(r[j]);
                            if (j < ncols) o[j] = bf ? f2bf(a) : f2h(a);
                        }
                    }
                }
            }
        }
    }

    // ---- teardown: drain what this CTA started, then free TMEM ----------
    __syncthreads();
    if (threadIdx.x == 0) {
        // TMA loads whose completion nobody observed (abort path only)
        const int issued = *(volatile int *)&ctl->issued;
        const int consumed = *(volatile int *)&ctl->consumed;
        for (int kb = consumed; kb < issued; kb++) {
            if (!mbar_wait(smem_u32(&ctl->full[kb % STAGES]), (uint32_t)(kb / STAGES) & 1u))
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
        }
    }
    if (threadIdx.x == 32) {
        // every MMA issued has retired once the final commit has arrived
        if (!mbar_wait(smem_u32(&ctl->accum), 0)) atomicExch(flag, HCT_B200_ERR_TIMEOUT);
    }
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------- basis

__global__ void basis_kernel(const double *__restrict__ tbl, uint64_t n, uint16_t *__restrict__ out,
                             uint64_t ld) {
    const uint64_t total = n * ld;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const double a0 = sqrt(1.0 / (double)n), a1 = sqrt(2.0 / (double)n);
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += stride) {
        const uint64_t i = idx / ld, k = idx - i * ld;
        uint16_t h = 0;
        if (k < n) {
            const uint64_t j = ((2 * i + 1) * k) % (4 * n);
            const double v = (k == 0 ? a0 : a1) * tbl[j];
            h = __half_as_ushort(__double2half(v));
        }
        out[idx] = h;
    }
}

// ---------------------------------------------------------------- host side

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// 2-D fp16 K-major operand: rows x K with row stride ld elements.
bool make_operand_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t K, uint64_t ld,
                      uint32_t box_rows) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {K, rows};
    cuuint64_t strides[1] = {ld * 2};
    cuuint32_t box[2] = {BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_basis(const double *d_cos_table, uint64_t n, half_bits *d_basis, uint64_t ld,
                         cudaStream_t s) {
    uint64_t total = n * ld;
    uint64_t g = (total + 255) / 256;
    if (g > 148ull * 64) g = 148ull * 64;
    if (g < 1) g = 1;
    basis_kernel<<<(unsigned)g, 256, 0, s>>>(d_cos_table, n, d_basis, ld);
    return cudaGetLastError();
}

cudaError_t launch_umma_gemm(const GemmArgs &a, cudaStream_t s) {
    if (a.M == 0 || a.N == 0) return cudaSuccess;
    if ((a.lda % 8) || (a.ldb % 8) || a.K == 0) return cudaErrorInvalidValue;
    if (a.M > 0x7fffffffull || a.N > 0x7fffffffull || a.K > 0x7fffffffull)
        return cudaErrorInvalidValue;
    alignas(64) CUtensorMap ta, tb;
    if (!make_operand_map(&ta, a.A, a.M, a.K, a.lda, BM)) return cudaErrorInvalidValue;
    if (!make_operand_map(&tb, a.B, a.N, a.K, a.ldb, BN)) return cudaErrorInvalidValue;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(umma_gemm_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SMEM_BYTES);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    const uint32_t m_tiles = (uint32_t)((a.M + BM - 1) / BM);
    const uint32_t n_tiles = (uint32_t)((a.N + BN - 1) / BN);
    const uint64_t ctas = (uint64_t)m_tiles * n_tiles;
    if (ctas > 0x7fffffffull) return cudaErrorInvalidValue;
    umma_gemm_kernel<<<(unsigned)ctas, THREADS, SMEM_BYTES, s>>>(
        ta, tb, (uint32_t)a.M, (uint32_t)a.N, (uint32_t)a.K, m_tiles, a.out, a.ldo, a.mode,
        a.out_dtype, a.d_flag);
    return cudaGetLastError();
}

}  // namespace hct
