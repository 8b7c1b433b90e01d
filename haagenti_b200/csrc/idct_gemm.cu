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
// The factored IDCT's two DFT stages (fdct.cu) run on dft_stage_t_kernel,
// a persistent variant: the DFT matrix stays resident in shared memory as
// the A operand, 128-row data tiles stream in as the B operand, TMEM is
// double-buffered so the epilogue of one tile overlaps the MMAs of the next,
// and 8 epilogue warps write each output as contiguous runs through a
// per-warp shared-memory transpose.
//
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
constexpr int BK = 64;  // 64 fp16 = 128 bytes = one 128B swizzle row
constexpr int MAX_STAGES = 4;
constexpr int A_TILE_BYTES = BM * BK * 2;
constexpr int THREADS = 192;

// Tile configuration: BN output columns per CTA (256 for the dense
// contraction, 128 for the short DFT stages so that two CTAs share an SM).
template <int BN_>
struct Cfg {
    static constexpr int STAGES = BN_ == 256 ? 4 : 3;
    static constexpr int B_TILE_BYTES = BN_ * BK * 2;
    static constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
    static constexpr int TMEM_COLS = BN_;
    static constexpr size_t SMEM_BYTES = 1024 /*align slack*/ + (size_t)STAGES * STAGE_BYTES + 256;
    // Instruction descriptor: kind::f16, A = B = fp16, D = f32, both K-major,
    // N = BN (bits 17..22 hold N>>3), M = 128 (bits 24..28 hold M>>4).
    static constexpr uint32_t IDESC =
        (1u << 4) | ((uint32_t)(BN_ >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
};

// Extra epilogue parameters of the factored-DCT stages (modes 2 and 3).
struct StageParams {
    uint32_t P, Q, H;
    uint32_t vec_out;  // output rows may be written with 16-byte stores
    uint64_t batch;
    const float2 *twiddle;
    float scale;
    // modes 4, 5 and 6: data tiles per k2 (mode 4), per m1 (mode 5) or per
    // column pair (mode 6), batch / 128
    uint32_t tiles_per_group;
    // mode 6: 64-wide k-blocks per column (2P <= 64 kbc)
    uint32_t kbc;
};

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

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar,
                                            int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// UMMA shared-memory descriptor, K-major, 128B swizzle: rows of 128 bytes,
// 8-row core groups 1024 bytes apart (SBO), LBO unused (1), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
}

// UMMA shared-memory descriptor, MN-major, 128B swizzle: atoms of 8 K-rows x
// 64 MN elements (128 bytes per row), 8-row K groups 1024 bytes apart (SBO),
// 64-element MN chunks lbo bytes apart (LBO), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
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
    uint64_t full[MAX_STAGES];
    uint64_t empty[MAX_STAGES];
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

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, uint32_t M, uint32_t N, uint32_t K,
                     uint32_t m_tiles, void *out, uint64_t ldo, int mode, int out_dtype,
                     int *flag, const StageParams sp) {
    using C = Cfg<BN>;
    constexpr int STAGES = C::STAGES;
    constexpr int STAGE_BYTES = C::STAGE_BYTES;
    constexpr int TMEM_COLS = C::TMEM_COLS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    SmemCtl *ctl = reinterpret_cast<SmemCtl *>(smem + (size_t)STAGES * STAGE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // mode 2 (DFT stage 1 with P > 128: a tall A against a short B) walks the
    // few n-tiles of one m-tile in consecutive CTAs, so that the A tile they
    // share is read from DRAM once and found in L2 by the others
    const uint32_t n_tiles = (N + BN - 1) / BN;
    const uint32_t m_tile = mode == 2 ? blockIdx.x / n_tiles : blockIdx.x % m_tiles;
    const uint32_t n_tile = mode == 2 ? blockIdx.x % n_tiles : blockIdx.x / m_tiles;
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
                    umma_f16(tmem, da + 2 * k, db + 2 * k, C::IDESC, (kb | k) != 0);
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
                if (mode == 2) {
                    // DFT stage 1 with P > 128 (the tiled path): this row is data
                    // row (b, k2), the columns are outputs 2 m1 + ri; the lanes of
                    // a warp (consecutive k2) store 32 consecutive complex values
                    const uint32_t Q = sp.Q, b = (uint32_t)row / Q, k2 = (uint32_t)row - b * Q;
                    uint32_t *g = reinterpret_cast<uint32_t *>(out);
                    // e^{2 pi i k2 m1 / H} for the chunk's first m1 (k2 m1 < Q P = H),
                    // then stepped by e^{2 pi i k2 / H} along m1
                    const uint32_t m1a = (uint32_t)col0 >> 1;
                    float2 tw = sp.twiddle[k2 * m1a];
                    const float2 st = sp.twiddle[k2];
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        if (j < ncols) {
                            const uint32_t m1 = m1a + (uint32_t)(j >> 1);
                            const float re = __uint_as_float(r[j]), im = __uint_as_float(r[j + 1]);
                            g[((uint64_t)m1 * sp.batch + b) * Q + k2] =
                                (uint32_t)f2h(re * tw.x - im * tw.y) |
                                ((uint32_t)f2h(re * tw.y + im * tw.x) << 16);
                        }
                        const float tx = tw.x * st.x - tw.y * st.y;
                        tw.y = tw.x * st.y + tw.y * st.x;
                        tw.x = tx;
                    }
                } else if (mode == 0) {
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

// ---------------------------------------------------------------- DFT stages
//
// Persistent kernel for the factored-DCT stages (modes 2-6): the stage's
// realified DFT matrix (at most 256 x 256 fp16; per k2 in mode 4 and per
// k2 pair in mode 6, reloaded when the tiles' group changes) is loaded into
// shared memory as the A operand; 128-line tiles of the data (the B
// operand) then stream through a ring of 64-column k-block stages, and two
// TMEM accumulators alternate so that the epilogue of one tile overlaps the
// TMA loads and MMAs of the next.  Two CTAs per SM for matrices of at most
// 128 rows and columns, one for up to 256; same warp roles and bounded waits
// as umma_gemm_kernel.
constexpr int TILE_SLOTS = 4;  // tiles announced ahead by the producer

struct StageCtl {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t wfull;
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint64_t tid_full[TILE_SLOTS];   // tile index published (producer arrives)
    uint64_t tid_empty[TILE_SLOTS];  // tile index read (MMA thread + 8 epilogue warps)
    uint64_t wempty;                 // mode 4: the MMAs that read the current W are done
    int tiles[TILE_SLOTS];           // tile index, -1 = no more tiles
    uint32_t tmem_base;
    int abort;
    int issued;    // ring slots the producer filled
    int consumed;  // ring slots whose "full" phase the MMA thread observed
    int w_issued;  // W loads the producer issued (one per k2 in mode 4, else one)
    int w_waited;  // W loads whose "wfull" phase the MMA thread observed
};

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

constexpr int STAGE_THREADS = 320;  // producer, MMA, 8 epilogue warps
constexpr int CTL_BYTES = 512;      // the StageCtl block at the end of shared memory
static_assert(sizeof(StageCtl) <= CTL_BYTES, "StageCtl outgrew its reserve");
#ifndef STAGE_RING2
#define STAGE_RING2 5  // ring slots of the one-CTA-per-SM configuration (MT = 2)
#endif

// ---------------------------------------------------------------- output-major stages

// DFT stage with the operands swapped: D^T = W . A^T, i.e. TMEM lane o holds
// DFT output o (the realified row of W) and TMEM column c holds data row
// r0 + c of the 128-row tile.  A lane's 32 columns are then 32 consecutive
// data rows of one output, which both stages store as contiguous runs:
//   stage 1: G[m1][b][k2] = G[m1 * batch * Q + r] for row r = (b, k2): the
//            lane pair (2 m1, 2 m1 + 1) trades halves of its chunk so that
//            each lane holds 16 complex values, twiddles them and writes
//            64 contiguous bytes;
//   stage 2: output row n(j, ri), j = m1 + P m2, columns b..b+31 of the
//            chunk (one m1 when batch % 32 == 0): 32 scaled values, 64 or
//            128 contiguous bytes.
// MT 128-row halves of W (2S <= 128 MT outputs) are resident in shared
// memory; the data tiles (128 rows x 64 K) stream through a TMA ring; per
// k-step one elected thread issues MT tcgen05 MMAs of M = 128, N = 128
// into a double-buffered TMEM accumulator.
// Per-warp staging of one 32-column chunk for coalesced stores: 2 KB per
// warp, its 16-byte pieces XOR-swizzled so that the 16-byte accesses of
// every quarter warp (on both the write and the read side) hit 8 distinct
// 4-bank groups:
//   stage 1: 16 slots of 128 bytes, piece p of slot s at (p ^ (s & 3));
//   stage 2: 32 rows of 64 bytes, piece p of row r at (p ^ ((r >> 1) & 3)).
constexpr int XWARP_BYTES = 2048;

template <int MT>
struct StageTCfg {
    static constexpr int WROWS = 128 * MT;
    static constexpr int KB_MAX = 2 * MT;              // K = 2S <= 128 MT
    static constexpr int W_KB_BYTES = WROWS * BK * 2;  // one 64-column k-block of W
    static constexpr int NT = 128;                     // data rows per tile (MMA N)
    static constexpr int B_TILE_BYTES = NT * BK * 2;
    static constexpr int RING = MT == 1 ? 3 : STAGE_RING2;
    static constexpr int TMEM_COLS = 2 * MT * NT;      // double-buffered
    static constexpr int X_BYTES = 8 * XWARP_BYTES;    // epilogue staging, 8 warps
    // MT = 1: 32 KB of W + 48 KB ring + 16 KB staging -> two CTAs per SM;
    // MT = 2: 128 KB of W + 80 KB ring + 16 KB staging -> one
    static constexpr size_t SMEM_BYTES = 1024 + (size_t)KB_MAX * W_KB_BYTES +
                                         (size_t)RING * B_TILE_BYTES + X_BYTES + CTL_BYTES;
    static constexpr uint32_t IDESC =
        (1u << 4) | ((uint32_t)(NT >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Stage 1 chunk: lane o = 2 m1 + ri holds columns rT..rT+31 of output o.
// After the pair exchange lane o owns 16 complex values of m1 (columns
// 16 ri..16 ri+15), twiddled and packed as fp16 pairs; the warp's 16 values
// of m1 (128 contiguous bytes of G) are then written by 8 lanes at a time.
// tw0: e^{2 pi i k2 m1 / H} of the chunk's first row (k2 = r1 mod Q), w: its
// step e^{2 pi i m1 / H}; both read from the table when have_tw is false.
__device__ __forceinline__ void stage1_chunk_t(const uint32_t (&r)[32], uint32_t o, uint32_t rT,
                                               uint32_t M, void *out, const StageParams &sp,
                                               uint8_t *xs, int lane, float2 tw0, float2 w0,
                                               bool have_tw) {
    const uint32_t m1 = o >> 1, ri = o & 1u;
    // even lane keeps columns 0..15 (needs the odd lane's Im), odd lane 16..31
    float re[16], im[16];
#pragma unroll
    for (int t = 0; t < 16; t++) {
        const uint32_t send = ri ? r[t] : r[16 + t];
        const float got = __uint_as_float(__shfl_xor_sync(0xffffffffu, send, 1));
        re[t] = ri ? got : __uint_as_float(r[t]);
        im[t] = ri ? __uint_as_float(r[16 + t]) : got;
    }
    const uint32_t Q = sp.Q;
    const uint32_t r1 = rT + 16 * ri;  // first data row of my 16
    uint32_t k2 = r1 % Q;
    // e^{2 pi i k2 m1 / H} (k2 m1 < H) and the step of k2 -> k2 + 1
    float2 tw = have_tw ? tw0 : sp.twiddle[m1 < sp.P ? k2 * m1 : 0];
    const float2 w = have_tw ? w0 : sp.twiddle[m1 < sp.P ? m1 : 0];
    uint32_t v[16];
    if (Q % 16 == 0) {  // my 16 rows start at a multiple of 16: one b, no wrap of k2
#pragma unroll
        for (int t = 0; t < 16; t++) {
            v[t] = pack_h2(re[t] * tw.x - im[t] * tw.y, re[t] * tw.y + im[t] * tw.x);
            const float tx = tw.x * w.x - tw.y * w.y;
            tw.y = tw.x * w.y + tw.y * w.x;
            tw.x = tx;
        }
    } else {
#pragma unroll
        for (int t = 0; t < 16; t++) {
            v[t] = pack_h2(re[t] * tw.x - im[t] * tw.y, re[t] * tw.y + im[t] * tw.x);
            if (++k2 == Q) {
                k2 = 0;
                tw = make_float2(1.0f, 0.0f);
            } else {
                const float tx = tw.x * w.x - tw.y * w.y;
                tw.y = tw.x * w.y + tw.y * w.x;
                tw.x = tx;
            }
        }
    }
    // stage: slot (lane >> 1) = the warp's m1 slot, 128 bytes = 32 complex
    const uint32_t wslot = (uint32_t)lane >> 1;
#pragma unroll
    for (int t = 0; t < 4; t++)
        *reinterpret_cast<uint4 *>(xs + wslot * 128 + (((4 * ri + t) ^ (wslot & 3)) * 16)) =
            make_uint4(v[4 * t], v[4 * t + 1], v[4 * t + 2], v[4 * t + 3]);
    __syncwarp();
    // 16 m1 rows of 128 bytes: lane writes piece (lane & 7) of rows (lane >> 3) + 4 i
    const uint32_t m1_base = (o - (uint32_t)lane) >> 1;
    const uint32_t piece = lane & 7;
    const uint32_t c0 = rT + 4 * piece;  // first data row of the piece (4 complex)
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t slot = (uint32_t)(lane >> 3) + 4 * i;
        const uint32_t mm = m1_base + slot;
        const uint4 val =
            *reinterpret_cast<const uint4 *>(xs + slot * 128 + ((piece ^ (slot & 3)) * 16));
        if (mm < sp.P) {
            uint32_t *g = reinterpret_cast<uint32_t *>(out) + (uint64_t)mm * sp.batch * Q + c0;
            if (c0 + 4 <= M) {
                *reinterpret_cast<uint4 *>(g) = val;  // 16-byte aligned (batch Q, c0 % 4 == 0)
            } else {
                const uint32_t e[4] = {val.x, val.y, val.z, val.w};
                for (int t = 0; t < 4; t++)
                    if (c0 + t < M) g[t] = e[t];
            }
        }
    }
    __syncwarp();
}

// Stage 1 chunk of modes 4 and 6 (twiddle folded into the per-k2 W): lane
// o = 2 m1 + ri holds 32 consecutive lines b0..b0+31 of one k2; each output
// row is 64 contiguous bytes of G[m1][k2][ri][b], the MN-major layout stage 2
// (mode 5) reads.  The warp's 32 rows are staged as 64-byte rows (16-byte
// pieces XOR-swizzled as in stage 2) and stored 4 lanes per row, so every
// store instruction writes 8 whole rows.
__device__ __forceinline__ void stage1_chunk_g(const uint32_t (&r)[32], uint32_t o, uint32_t k2,
                                               uint64_t b0, void *out, const StageParams &sp,
                                               uint8_t *xs, int lane) {
    const uint32_t wsw = ((uint32_t)lane >> 1) & 3;
#pragma unroll
    for (int t = 0; t < 4; t++)
        *reinterpret_cast<uint4 *>(xs + lane * 64 + ((t ^ wsw) * 16)) = make_uint4(
            pack_h2(__uint_as_float(r[8 * t]), __uint_as_float(r[8 * t + 1])),
            pack_h2(__uint_as_float(r[8 * t + 2]), __uint_as_float(r[8 * t + 3])),
            pack_h2(__uint_as_float(r[8 * t + 4]), __uint_as_float(r[8 * t + 5])),
            pack_h2(__uint_as_float(r[8 * t + 6]), __uint_as_float(r[8 * t + 7])));
    __syncwarp();
    const uint32_t o_base = o - (uint32_t)lane, piece = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const uint32_t row = (uint32_t)(lane >> 2) + 8 * i;
        const uint32_t oo = o_base + row, m1 = oo >> 1, ri = oo & 1u;
        const uint4 val =
            *reinterpret_cast<const uint4 *>(xs + row * 64 + ((piece ^ ((row >> 1) & 3)) * 16));
        if (m1 < sp.P)
            *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) +
                                       (((uint64_t)m1 * sp.Q + k2) * 2 + ri) * sp.batch + b0 +
                                       8 * piece) = val;
    }
    __syncwarp();
}

// Stage 2 chunk: lane o = 2 m2 + ri holds columns rT..rT+31 = rows (m1, b).
// With batch % 32 == 0 the chunk is one m1 and b0..b0+31: each output row
// n(j, ri) receives 32 contiguous values, staged as 64-byte rows (two
// rounds for f32) and written 4 lanes per row.
template <int DT>
__device__ __forceinline__ void stage2_chunk_t(const uint32_t (&r)[32], uint32_t o, uint32_t rT,
                                               uint32_t M, void *out, uint64_t ldo,
                                               const StageParams &sp, uint8_t *xs, int lane) {
    const uint32_t batch = (uint32_t)sp.batch, half = sp.H / 2;
    if (batch % 32 == 0 && sp.vec_out) {
        if (rT >= M) return;  // warp-uniform
        const uint32_t m1 = rT / batch, b0 = rT - m1 * batch;
        const float sc = sp.scale;
        constexpr int PARTS = DT == HCT_B200_F32 ? 2 : 1;  // 64 bytes of a row per part
        constexpr int PER = 32 / PARTS;                    // values per part
        const uint32_t o_base = o - (uint32_t)lane, piece = lane & 3;
        uint32_t nrow[4];
        bool ok[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t oo = o_base + (uint32_t)(lane >> 2) + 8 * i, m2 = oo >> 1, ri = oo & 1u;
            const uint32_t j = m1 + sp.P * m2;
            ok[i] = m2 < sp.Q;
            nrow[i] = j < half ? 4 * j + 2 * ri : 4 * (sp.H - 1 - j) + 3 - 2 * ri;
        }
#pragma unroll
        for (int part = 0; part < PARTS; part++) {
            uint8_t *xw = xs + lane * 64;
            const uint32_t wsw = ((uint32_t)lane >> 1) & 3;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                uint32_t p[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    if (DT == HCT_B200_F32) {
                        p[u] = __float_as_uint(__uint_as_float(r[PER * part + 4 * t + u]) * sc);
                    } else {
                        const float a = __uint_as_float(r[8 * t + 2 * u]) * sc;
                        const float b = __uint_as_float(r[8 * t + 2 * u + 1]) * sc;
                        p[u] = DT == HCT_B200_BF16 ? pack_bf2(a, b) : pack_h2(a, b);
                    }
                }
                *reinterpret_cast<uint4 *>(xw + ((t ^ wsw) * 16)) = make_uint4(p[0], p[1], p[2], p[3]);
            }
            __syncwarp();
            // rows (lane >> 2) + 8 i of the staging, 16-byte piece (lane & 3)
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint32_t row = (uint32_t)(lane >> 2) + 8 * i;
                const uint4 val = *reinterpret_cast<const uint4 *>(
                    xs + row * 64 + ((piece ^ ((row >> 1) & 3)) * 16));
                if (ok[i]) {
                    if (DT == HCT_B200_F32)
                        *reinterpret_cast<uint4 *>(reinterpret_cast<float *>(out) +
                                                   (uint64_t)nrow[i] * ldo + b0 + PER * part +
                                                   4 * piece) = val;
                    else
                        *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) +
                                                   (uint64_t)nrow[i] * ldo + b0 + 8 * piece) = val;
                }
            }
            __syncwarp();
        }
        return;
    }
    const uint32_t m2 = o >> 1, ri = o & 1u;
    if (m2 >= sp.Q) return;
    for (int t = 0; t < 32; t++) {
        const uint32_t rr = rT + t;
        if (rr >= M) break;
        const uint32_t m1 = rr / batch, b = rr - m1 * batch;
        const uint32_t j = m1 + sp.P * m2;
        const uint32_t n = j < half ? 4 * j + 2 * ri : 4 * (sp.H - 1 - j) + 3 - 2 * ri;
        const float v = __uint_as_float(r[t]) * sp.scale;
        const uint64_t idx = (uint64_t)n * ldo + b;
        if (DT == HCT_B200_F32) reinterpret_cast<float *>(out)[idx] = v;
        else if (DT == HCT_B200_BF16) reinterpret_cast<uint16_t *>(out)[idx] = f2bf(v);
        else reinterpret_cast<uint16_t *>(out)[idx] = f2h(v);
    }
}

template <int MT>
__global__ void __launch_bounds__(STAGE_THREADS, MT == 1 ? 2 : 1)
    dft_stage_t_kernel(const __grid_constant__ CUtensorMap tmD,
                       const __grid_constant__ CUtensorMap tmW, uint32_t M, uint32_t K,
                       uint32_t m_tiles, void *out, uint64_t ldo, int mode, int out_dtype,
                       int *flag, const StageParams sp, uint32_t *tile_counter) {
    using SC = StageTCfg<MT>;
    constexpr int RING = SC::RING;
    constexpr int NT = SC::NT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *w_smem = smem;
    uint8_t *d_smem = smem + (size_t)SC::KB_MAX * SC::W_KB_BYTES;
    uint8_t *x_smem = d_smem + (size_t)RING * SC::B_TILE_BYTES;
    StageCtl *ctl = reinterpret_cast<StageCtl *>(x_smem + SC::X_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kbs = (int)((K + BK - 1) / BK);

    if (threadIdx.x == 0) {
        for (int s = 0; s < RING; s++) {
            mbar_init(smem_u32(&ctl->full[s]), 1);
            mbar_init(smem_u32(&ctl->empty[s]), 1);
        }
        mbar_init(smem_u32(&ctl->wfull), 1);
        for (int b = 0; b < 2; b++) {
            mbar_init(smem_u32(&ctl->tfull[b]), 1);
            mbar_init(smem_u32(&ctl->tempty[b]), 8);  // one arrive per epilogue warp
        }
        mbar_init(smem_u32(&ctl->drain), 1);
        mbar_init(smem_u32(&ctl->wempty), 1);
        for (int t = 0; t < TILE_SLOTS; t++) {
            mbar_init(smem_u32(&ctl->tid_full[t]), 1);
            mbar_init(smem_u32(&ctl->tid_empty[t]), 9);  // MMA thread + 8 epilogue warps
        }
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        ctl->w_issued = 0;
        ctl->w_waited = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    // mode 4: each CTA takes a contiguous range of tiles, so that the k2 of
    // consecutive tiles (and with it the W in shared memory) rarely changes
    const uint32_t per_cta = (m_tiles + gridDim.x - 1) / gridDim.x;
    const uint32_t tpg = sp.tiles_per_group;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&ctl->tmem_base)),
                     "r"(SC::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmD))
                         : "memory");
            const uint32_t wb = smem_u32(&ctl->wfull);
            // modes 4 and 6: the per-group W is loaded when the group of the
            // tiles changes
            const bool wgroup = mode == 4 || mode == 6;
            if (!wgroup) {
                mbar_expect_tx(wb, (uint32_t)(kbs * SC::W_KB_BYTES));
                for (int kb = 0; kb < kbs; kb++)
                    tma_load_2d(smem_u32(w_smem + (size_t)kb * SC::W_KB_BYTES), &tmW, wb, kb * BK,
                                0);
                *(volatile int *)&ctl->w_issued = 1;
            }
            int it = 0, w_issued = 0;
            uint32_t cur_g = 0xffffffffu;
            for (uint32_t i = 0;; i++) {
                // the next tile: the CTA's range (mode 4), the counter, or every
                // gridDim.x-th
                const uint32_t t =
                    wgroup ? (i < per_cta ? blockIdx.x * per_cta + i : m_tiles)
                           : (tile_counter ? atomicAdd(tile_counter, 1u) : blockIdx.x + i * gridDim.x);
                const int slot = (int)(i % TILE_SLOTS);
                if (*(volatile int *)&ctl->abort) break;
                if (!mbar_wait(smem_u32(&ctl->tid_empty[slot]), ((i / TILE_SLOTS) & 1u) ^ 1u)) {
                    atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                    atomicExch(&ctl->abort, 1);
                    break;
                }
                *(volatile int *)&ctl->tiles[slot] = t < m_tiles ? (int)t : -1;
                mbar_arrive(smem_u32(&ctl->tid_full[slot]));
                if (t >= m_tiles) break;
                const int r0 = (int)(t * NT);
                if (wgroup && t / tpg != cur_g) {
                    // the previous W must no longer be read by any MMA
                    if (w_issued > 0 &&
                        !mbar_wait(smem_u32(&ctl->wempty), (uint32_t)(w_issued - 1) & 1u)) {
                        atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                        atomicExch(&ctl->abort, 1);
                        break;
                    }
                    cur_g = t / tpg;
                    mbar_expect_tx(wb, (uint32_t)(kbs * SC::W_KB_BYTES));
                    for (int kb = 0; kb < kbs; kb++)
                        tma_load_2d(smem_u32(w_smem + (size_t)kb * SC::W_KB_BYTES), &tmW, wb,
                                    kb * BK, (int)(cur_g * SC::WROWS));
                    *(volatile int *)&ctl->w_issued = ++w_issued;
                }
                bool stop = false;
                for (int kb = 0; kb < kbs; kb++, it++) {
                    const int s = it % RING;
                    const uint32_t ph = (uint32_t)(it / RING) & 1u;
                    if (*(volatile int *)&ctl->abort) { stop = true; break; }
                    if (!mbar_wait(smem_u32(&ctl->empty[s]), ph ^ 1u)) {
                        atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                        atomicExch(&ctl->abort, 1);
                        stop = true;
                        break;
                    }
                    const uint32_t fb = smem_u32(&ctl->full[s]);
                    mbar_expect_tx(fb, SC::B_TILE_BYTES);
                    uint8_t *slot_p = d_smem + (size_t)s * SC::B_TILE_BYTES;
                    if (mode == 5) {
                        // MN-major tile: K rows (k2, ri) of m1, 128 b as two 64-wide boxes
                        const uint32_t m1 = t / tpg, b0 = (t - m1 * tpg) * NT;
                        const int y = (int)(m1 * K) + kb * BK;
                        tma_load_2d(smem_u32(slot_p), &tmD, fb, (int)b0, y);
                        tma_load_2d(smem_u32(slot_p + SC::B_TILE_BYTES / 2), &tmD, fb, (int)b0 + 64,
                                    y);
                    } else if (mode == 6) {
                        // k-block kb: 64 values of column u (first kbc blocks) or of
                        // column (Q - u) mod Q, for 128 lines
                        const uint32_t u = t / tpg, n0 = (t - u * tpg) * NT;
                        const uint32_t blk = (uint32_t)kb / sp.kbc;
                        const uint32_t col = blk == 0 ? u : (sp.Q - u) % sp.Q;
                        tma_load_3d(smem_u32(slot_p), &tmD, fb, (int)(((uint32_t)kb - blk * sp.kbc) * BK),
                                    (int)col, (int)n0);
                    } else {
                        tma_load_2d(smem_u32(slot_p), &tmD, fb, kb * BK, r0);
                    }
                    *(volatile int *)&ctl->issued = it + 1;
                }
                if (stop) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            int w_waited = 0;
            uint32_t cur_g = 0xffffffffu;
            const bool wgroup = mode == 4 || mode == 6;
            if (!wgroup) {
                ok = mbar_wait(smem_u32(&ctl->wfull), 0);
                if (ok) *(volatile int *)&ctl->w_waited = w_waited = 1;
            }
            const uint32_t idesc = mode == 5 ? SC::IDESC | (1u << 16) : SC::IDESC;  // B MN-major
            int it = 0;
            for (uint32_t i = 0; ok; i++) {
                const int buf = (int)(i & 1u);
                const uint32_t use = i >> 1;
                if (*(volatile int *)&ctl->abort) break;
                const int slot = (int)(i % TILE_SLOTS);
                if (!mbar_wait(smem_u32(&ctl->tid_full[slot]), (i / TILE_SLOTS) & 1u)) {
                    ok = false;
                    break;
                }
                const int tile = *(volatile int *)&ctl->tiles[slot];
                mbar_arrive(smem_u32(&ctl->tid_empty[slot]));
                if (tile < 0) break;
                if (wgroup && (uint32_t)tile / tpg != cur_g) {
                    if (!mbar_wait(smem_u32(&ctl->wfull), (uint32_t)w_waited & 1u)) {
                        ok = false;
                        break;
                    }
                    *(volatile int *)&ctl->w_waited = ++w_waited;
                    cur_g = (uint32_t)tile / tpg;
                }
                if (!mbar_wait(smem_u32(&ctl->tempty[buf]), (use & 1u) ^ 1u)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + (uint32_t)(buf * MT * NT);
                for (int kb = 0; kb < kbs; kb++, it++) {
                    const int s = it % RING;
                    const uint32_t ph = (uint32_t)(it / RING) & 1u;
                    if (!mbar_wait(smem_u32(&ctl->full[s]), ph)) { ok = false; break; }
                    *(volatile int *)&ctl->consumed = it + 1;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint32_t sb = smem_u32(d_smem + (size_t)s * SC::B_TILE_BYTES);
                    // K-major: +32 bytes per 16 K; MN-major: +16 rows of 128 bytes
                    const uint64_t db = mode == 5 ? umma_desc_sw128_mn(sb, SC::B_TILE_BYTES / 2)
                                                  : umma_desc_sw128(sb);
                    const uint32_t dstep = mode == 5 ? 128u : 2u;
#pragma unroll
                    for (int hh = 0; hh < MT; hh++) {
                        // rows 128 hh.. of the k-block: 16 core groups of 1 KB further
                        const uint64_t da = umma_desc_sw128(
                            smem_u32(w_smem + (size_t)kb * SC::W_KB_BYTES + (size_t)hh * 128 * 128));
#pragma unroll
                        for (int k = 0; k < BK / 16; k++)
                            umma_f16(d + (uint32_t)(hh * NT), da + 2 * k, db + dstep * k, idesc,
                                     (kb | k) != 0);
                    }
                    umma_commit(smem_u32(&ctl->empty[s]));
                }
                if (!ok) break;
                umma_commit(smem_u32(&ctl->tfull[buf]));
                if (wgroup) {
                    // the last tile of this W: release it to the producer once read
                    const uint32_t nx = (uint32_t)tile + 1;
                    const bool last = i + 1 >= per_cta || nx >= m_tiles || nx / tpg != cur_g;
                    if (last) umma_commit(smem_u32(&ctl->wempty));
                }
            }
            if (!ok) {
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                atomicExch(&ctl->abort, 1);
            }
            umma_commit(smem_u32(&ctl->drain));  // arrives once every MMA above retired
        }
    } else {
        // 8 epilogue warps: TMEM lane quarter q = warp % 4; h = column half
        // (MT = 1) or W half (MT = 2)
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;
        const int hh = MT == 2 ? h : 0;
        const int c_begin = MT == 2 ? 0 : 64 * h;  // my columns: c_begin .. c_begin + 32 NCH
        const uint32_t o = (uint32_t)(128 * hh + 32 * q + lane);  // my DFT output
        uint8_t *xs = x_smem + (warp - 2) * XWARP_BYTES;
        // stage 1: the twiddle step of my output, and, when Q divides the tile
        // height (k2 of a chunk's first row is then the same in every tile),
        // the first twiddle of each of my chunks
        constexpr int NCH = MT == 2 ? NT / 32 : 2;
        float2 tw_first[NCH], tw_step = make_float2(1.0f, 0.0f);
        const bool tw_fixed = mode == 2 && NT % sp.Q == 0;
        if (mode == 2) {
            const uint32_t m1 = o >> 1, ri = o & 1u;
            const bool live = m1 < sp.P;
            tw_step = sp.twiddle[live ? m1 : 0];
#pragma unroll
            for (int ci = 0; ci < NCH; ci++) {
                const uint32_t k2 = ((uint32_t)c_begin + 32 * ci + 16 * ri) % sp.Q;
                tw_first[ci] = tw_fixed && live ? sp.twiddle[k2 * m1] : make_float2(1.0f, 0.0f);
            }
        }
        for (uint32_t i = 0;; i++) {
            const int buf = (int)(i & 1u);
            const uint32_t use = i >> 1;
            const int slot = (int)(i % TILE_SLOTS);
            if (!mbar_wait(smem_u32(&ctl->tid_full[slot]), (i / TILE_SLOTS) & 1u)) {
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                atomicExch(&ctl->abort, 1);
                break;
            }
            const int tile = *(volatile int *)&ctl->tiles[slot];
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctl->tid_empty[slot]));
            if (tile < 0) break;
            if (!mbar_wait(smem_u32(&ctl->tfull[buf]), use & 1u)) {
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                atomicExch(&ctl->abort, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t r0 = (uint32_t)tile * NT;
            const uint32_t taddr =
                tmem + (uint32_t)(buf * MT * NT + hh * NT) + ((uint32_t)(q * 32) << 16);
            // modes 4 and 6: the k2 of my outputs and the tile's first line
            const uint32_t grp = (uint32_t)tile / tpg;
            const uint64_t line0 = (uint64_t)((uint32_t)tile - grp * tpg) * NT;
            uint32_t k2 = grp;
            bool live = true;
            if (mode == 6) {
                // W half hh computes k2 = u (hh = 0) or Q - u (hh = 1); the
                // pairs u = 0 and u = Q/2 have no second k2
                k2 = hh ? sp.Q - grp : grp;
                live = hh == 0 || (grp != 0 && 2 * grp != sp.Q);
            }
#pragma unroll
            for (int ci = 0; ci < NCH; ci++) {
                const int c = c_begin + 32 * ci;
                uint32_t r[32];
                if (!live) break;  // warp-uniform
                tmem_ld32(taddr + (uint32_t)c, r);
                if (mode == 4 || mode == 6) {
                    stage1_chunk_g(r, mode == 6 ? o - 128u * (uint32_t)hh : o, k2, line0 + c, out,
                                   sp, xs, lane);
                } else if (mode == 2) {
                    stage1_chunk_t(r, o, r0 + c, M, out, sp, xs, lane, tw_first[ci], tw_step,
                                   tw_fixed);
                } else if (out_dtype == HCT_B200_F16) {
                    stage2_chunk_t<HCT_B200_F16>(r, o, r0 + c, M, out, ldo, sp, xs, lane);
                } else if (out_dtype == HCT_B200_BF16) {
                    stage2_chunk_t<HCT_B200_BF16>(r, o, r0 + c, M, out, ldo, sp, xs, lane);
                } else {
                    stage2_chunk_t<HCT_B200_F32>(r, o, r0 + c, M, out, ldo, sp, xs, lane);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctl->tempty[buf]));
        }
    }

    // ---- teardown: drain this CTA's copies and MMAs, then free TMEM ------
    __syncthreads();
    if (threadIdx.x == 0) {
        // a W load nobody waited for (abort path): at most the latest one
        const int wi = *(volatile int *)&ctl->w_issued, ww = *(volatile int *)&ctl->w_waited;
        if (ww < wi && !mbar_wait(smem_u32(&ctl->wfull), (uint32_t)(wi - 1) & 1u))
            atomicExch(flag, HCT_B200_ERR_TIMEOUT);
        const int issued = *(volatile int *)&ctl->issued;
        const int consumed = *(volatile int *)&ctl->consumed;
        for (int it = consumed; it < issued; it++)
            if (!mbar_wait(smem_u32(&ctl->full[it % RING]), (uint32_t)(it / RING) & 1u))
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
    }
    if (threadIdx.x == 32) {
        if (!mbar_wait(smem_u32(&ctl->drain), 0)) atomicExch(flag, HCT_B200_ERR_TIMEOUT);
    }
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(SC::TMEM_COLS)
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

// 3-D fp16 operand of mode 6: lines of `cols` columns of `len` values each
// (line stride ld elements), read as boxes of 64 values of one column for
// box_lines lines (128-byte rows: the K-major, 128B-swizzled layout).
bool make_column_map(CUtensorMap *map, const void *base, uint64_t len, uint64_t cols,
                     uint64_t lines, uint64_t ld, uint32_t box_lines) {
    EncodeTiledFn enc = get_encode_fn();
    if (!enc) return false;
    cuuint64_t dims[3] = {len, cols, lines};
    cuuint64_t strides[2] = {len * 2, ld * 2};
    cuuint32_t box[3] = {BK, 1, box_lines};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims,
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

namespace {

template <int BN>
cudaError_t launch_bn(const GemmArgs &a, cudaStream_t s) {
    using C = Cfg<BN>;
    alignas(64) CUtensorMap ta, tb;
    if (!make_operand_map(&ta, a.A, a.M, a.K, a.lda, BM)) return cudaErrorInvalidValue;
    if (!make_operand_map(&tb, a.B, a.N, a.K, a.ldb, BN)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(umma_gemm_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)C::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const uint32_t m_tiles = (uint32_t)((a.M + BM - 1) / BM);
    const uint32_t n_tiles = (uint32_t)((a.N + BN - 1) / BN);
    const uint64_t ctas = (uint64_t)m_tiles * n_tiles;
    if (ctas > 0x7fffffffull) return cudaErrorInvalidValue;
    StageParams sp{a.P, a.Q, a.H, 0, a.batch, reinterpret_cast<const float2 *>(a.twiddle), a.scale,
                   0};
    umma_gemm_kernel<BN><<<(unsigned)ctas, THREADS, C::SMEM_BYTES, s>>>(
        ta, tb, (uint32_t)a.M, (uint32_t)a.N, (uint32_t)a.K, m_tiles, a.out, a.ldo, a.mode,
        a.out_dtype, a.d_flag, sp);
    return cudaGetLastError();
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
    }
    return n;
}

template <int MT>
cudaError_t launch_stage_t(const GemmArgs &a, cudaStream_t s) {
    using SC = StageTCfg<MT>;
    if (a.K > (uint64_t)SC::KB_MAX * BK || a.N > (uint64_t)SC::WROWS) return cudaErrorInvalidValue;
    if ((a.mode == 4 || a.mode == 5 || a.mode == 6) && a.batch % SC::NT)
        return cudaErrorInvalidValue;
    if (a.mode == 5 && a.K % BK) return cudaErrorInvalidValue;  // K-row boxes stay in one m1
    uint32_t kbc = 0;
    if (a.mode == 6) {
        // two columns of 2P values per line, each in kbc 64-wide k-blocks; the
        // first box of a column lies inside it, 16-byte strides
        kbc = (2 * a.P + BK - 1) / BK;
        if (MT != 2 || 2 * a.P < (uint32_t)BK || 2 * a.P > 2u * BK || a.P % 4 || a.Q % 2 ||
            a.K != 2ull * kbc * BK || a.M != (uint64_t)(a.Q / 2 + 1) * a.batch || a.lda % 8 ||
            a.lda < 2ull * a.P * a.Q)
            return cudaErrorInvalidValue;
    }
    alignas(64) CUtensorMap td, tw;
    if (a.mode == 5) {
        // G[m1][k2][ri][b]: P * 2Q rows of batch b, read as 64 x 64 MN-major boxes
        if (!make_operand_map(&td, a.A, (uint64_t)a.P * a.K, a.batch, a.lda, BK))
            return cudaErrorInvalidValue;
    } else if (a.mode == 6) {
        // T'[n][k2][r]: batch lines of lda values, a line's Q columns of 2P
        if (!make_column_map(&td, a.A, 2ull * a.P, a.Q, a.batch, a.lda, SC::NT))
            return cudaErrorInvalidValue;
    } else if (!make_operand_map(&td, a.A, a.M, a.K, a.lda, SC::NT)) {
        return cudaErrorInvalidValue;
    }
    // modes 4 and 6: the table of per-group matrices, WROWS rows each
    const uint64_t w_rows = a.mode == 4   ? (uint64_t)a.Q * SC::WROWS
                            : a.mode == 6 ? (uint64_t)(a.Q / 2 + 1) * SC::WROWS
                                          : a.N;
    if (!make_operand_map(&tw, a.B, w_rows, a.K, a.ldb, SC::WROWS)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(dft_stage_t_kernel<MT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SC::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const uint64_t m_tiles = (a.M + SC::NT - 1) / SC::NT;
    if (m_tiles > 0x7fffffffull) return cudaErrorInvalidValue;
    const uint64_t per_sm = MT == 1 ? 2 : 1;  // shared memory and TMEM
    const uint32_t grid = (uint32_t)std::min<uint64_t>(m_tiles, per_sm * (uint64_t)sm_count());
    // 16-byte output runs need an aligned base and row stride (stage 2)
    const uint32_t vec = ((uintptr_t)a.out % 16 == 0) && (a.ldo % 8 == 0);
    StageParams sp{a.P, a.Q, a.H, vec, a.batch, reinterpret_cast<const float2 *>(a.twiddle),
                   a.scale, (uint32_t)(a.batch / SC::NT), kbc};
    if (a.tile_counter) {
        e = cudaMemsetAsync(a.tile_counter, 0, sizeof(uint32_t), s);
        if (e != cudaSuccess) return e;
    }
    dft_stage_t_kernel<MT><<<grid, STAGE_THREADS, SC::SMEM_BYTES, s>>>(
        td, tw, (uint32_t)a.M, (uint32_t)a.K, (uint32_t)m_tiles, a.out, a.ldo, a.mode,
        a.out_dtype, a.d_flag, sp, a.tile_counter);
    return cudaGetLastError();
}

}  // namespace

uint32_t stage_w_rows(uint64_t N, uint64_t K) { return N <= 128 && K <= 128 ? 128u : 256u; }

cudaError_t launch_umma_gemm(const GemmArgs &a, cudaStream_t s) {
    if (a.M == 0 || a.N == 0) return cudaSuccess;
    if ((a.lda % 8) || (a.ldb % 8) || a.K == 0) return cudaErrorInvalidValue;
    if (a.M > 0x7fffffffull || a.N > 0x7fffffffull || a.K > 0x7fffffffull)
        return cudaErrorInvalidValue;
    if ((a.mode == 2 || a.mode == 3) &&
        (!a.P || !a.Q || !a.batch || (a.mode == 3 && (a.N > 256 || a.K > 256)) ||
         (a.mode == 2 && (!a.twiddle || (a.N & 1)))))
        return cudaErrorInvalidValue;
    if (a.mode == 2 || a.mode == 3) {
        if (a.N <= 128 && a.K <= 128) return launch_stage_t<1>(a, s);
        if (a.N <= 256 && a.K <= 256) return launch_stage_t<2>(a, s);
        // stage 1 with P > 128: output tiles of the general contraction
        return launch_bn<256>(a, s);
    }
    if (a.mode == 4 || a.mode == 5) {
        if (!a.P || !a.Q || !a.batch || a.N > 256 || a.K > 256) return cudaErrorInvalidValue;
        if (stage_w_rows(a.N, a.K) == 128) return launch_stage_t<1>(a, s);
        return launch_stage_t<2>(a, s);
    }
    if (a.mode == 6) {
        if (!a.P || !a.Q || !a.batch || a.N != 256 || a.K > 256) return cudaErrorInvalidValue;
        return launch_stage_t<2>(a, s);
    }
    if (a.N <= 128) return launch_bn<128>(a, s);
    return launch_bn<256>(a, s);
}

}  // namespace hct
