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
    uint32_t pad;
    uint64_t batch;
    const float2 *twiddle;
    float scale;
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

// UMMA shared-memory descriptor, K-major, 128B swizzle: rows of 128 bytes,
// 8-row core groups 1024 bytes apart (SBO), LBO unused (1), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) | (1ull << 46) |
           (2ull << 61);
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

// Epilogue of the factored-DCT stages for one 32-column chunk of a TMEM row
// (fp32 accumulator values r[0..31] of D row `row`, columns col0..col0+31).
//   mode 2 (stage 1): row = (b, k2); column pair (2 m1, 2 m1 + 1) = complex
//           output m1, multiplied by twiddle[k2 * m1] and stored as an fp16
//           pair at G[(m1 * batch + b) * Q + k2].
//   mode 3 (stage 2): row = (m1, b); column pair (2 m2, 2 m2 + 1) = z[j],
//           j = m1 + P m2, scaled; Re/Im go to output rows 4j, 4j+2
//           (j < H/2) or 4(H-1-j)+3, 4(H-1-j)+1, at column b.
// Stage 1 (mode 2), one 32-column chunk = complex outputs m1 in
// [m1_0, m1_0 + 16) of row (b, k2).  `g` points at G[(0 * batch + b) * Q + k2]
// (fp16 pairs as u32); consecutive m1 are `stride` = batch * Q apart.
// The twiddles e^{2 pi i k2 m1 / H} run by recurrence from the table entry
// at m1_0 (16 steps of an fp32 complex product).
__device__ __forceinline__ void stage1_chunk(const uint32_t (&r)[32], uint32_t *g, uint64_t stride,
                                             uint32_t m1_0, uint32_t P, float2 t, float2 w) {
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const uint32_t m1 = m1_0 + j;
        if (m1 < P) {
            const float re = __uint_as_float(r[2 * j]), im = __uint_as_float(r[2 * j + 1]);
            const float yr = re * t.x - im * t.y, yi = re * t.y + im * t.x;
            g[(uint64_t)m1 * stride] = (uint32_t)f2h(yr) | ((uint32_t)f2h(yi) << 16);
        }
        const float tx = t.x * w.x - t.y * w.y;
        t.y = t.x * w.y + t.y * w.x;
        t.x = tx;
    }
}

// Stage 2 (mode 3), one chunk = z[j] for m2 in [m2_0, m2_0 + 16) of row
// (m1, b), j = m1 + P m2; output rows per the Makhoul quartet map, column b.
template <int DT>
__device__ __forceinline__ void stage2_chunk(const uint32_t (&r)[32], void *out, uint64_t ldo,
                                             uint32_t b, uint32_t m1, uint32_t m2_0,
                                             const StageParams &sp) {
    const uint32_t half = sp.H / 2;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        const uint32_t m2 = m2_0 + j;
        if (m2 < sp.Q) {
            const uint32_t jj = m1 + sp.P * m2;
            const uint32_t n_re = jj < half ? 4 * jj : 4 * (sp.H - 1 - jj) + 3;
            const uint32_t n_im = jj < half ? n_re + 2 : n_re - 2;
            const float zr = __uint_as_float(r[2 * j]) * sp.scale;
            const float zi = __uint_as_float(r[2 * j + 1]) * sp.scale;
            const uint64_t ore = (uint64_t)n_re * ldo + b, oim = (uint64_t)n_im * ldo + b;
            if (DT == HCT_B200_F32) {
                reinterpret_cast<float *>(out)[ore] = zr;
                reinterpret_cast<float *>(out)[oim] = zi;
            } else if (DT == HCT_B200_BF16) {
                reinterpret_cast<uint16_t *>(out)[ore] = f2bf(zr);
                reinterpret_cast<uint16_t *>(out)[oim] = f2bf(zi);
            } else {
                reinterpret_cast<uint16_t *>(out)[ore] = f2h(zr);
                reinterpret_cast<uint16_t *>(out)[oim] = f2h(zi);
            }
        }
    }
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

// ---------------------------------------------------------------- DFT stages
//
// Persistent kernel for the factored-DCT stages (modes 2 and 3): the stage's
// realified DFT matrix (the B operand, at most 256 x 256 fp16) is loaded into
// shared memory once per CTA; 128-row tiles of the data (the A operand) then
// stream through a ring of 64-column k-block stages, and two TMEM
// accumulators alternate so that the epilogue of one tile overlaps the TMA
// loads and MMAs of the next.  One CTA per SM; same warp roles and bounded
// waits as umma_gemm_kernel.
template <int BN>
struct StageCfg {
    static constexpr int KB_MAX = BN / 64;           // K <= BN (K = N = 2 * DFT size)
    static constexpr int W_KB_BYTES = BN * BK * 2;   // one 64-column k-block of W
    // BN = 128: 32 KB of W + 4 x 16 KB ring -> two CTAs per SM
    static constexpr int RING = BN == 256 ? 5 : 4;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr size_t SMEM_BYTES =
        1024 + (size_t)KB_MAX * W_KB_BYTES + (size_t)RING * A_TILE_BYTES + 256;
};

struct StageCtl {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t wfull;
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
    int issued;    // ring slots the producer filled
    int consumed;  // ring slots whose "full" phase the MMA thread observed
    int w_waited;  // the MMA thread observed the W load
};

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

constexpr int STAGE_THREADS = 320;  // producer, MMA, 8 epilogue warps

template <int BN>
__global__ void __launch_bounds__(STAGE_THREADS, 1)
    dft_stage_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, uint32_t M, uint32_t N, uint32_t K,
                     uint32_t m_tiles, void *out, uint64_t ldo, int mode, int out_dtype, int *flag,
                     const StageParams sp) {
    using SC = StageCfg<BN>;
    constexpr int RING = SC::RING;
    constexpr uint32_t IDESC = Cfg<BN>::IDESC;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *w_smem = smem;
    uint8_t *a_smem = smem + (size_t)SC::KB_MAX * SC::W_KB_BYTES;
    StageCtl *ctl = reinterpret_cast<StageCtl *>(a_smem + (size_t)RING * A_TILE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kbs = (int)((K + BK - 1) / BK);
    const uint32_t my_tiles =
        blockIdx.x < m_tiles ? (m_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

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
        ctl->abort = 0;
        ctl->issued = 0;
        ctl->consumed = 0;
        ctl->w_waited = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
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
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA))
                         : "memory");
            const uint32_t wb = smem_u32(&ctl->wfull);
            mbar_expect_tx(wb, (uint32_t)(kbs * SC::W_KB_BYTES));
            for (int kb = 0; kb < kbs; kb++)
                tma_load_2d(smem_u32(w_smem + (size_t)kb * SC::W_KB_BYTES), &tmB, wb, kb * BK, 0);
            int it = 0;
            for (uint32_t i = 0; i < my_tiles; i++) {
                const int m0 = (int)((blockIdx.x + i * gridDim.x) * BM);
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
                    mbar_expect_tx(fb, A_TILE_BYTES);
                    tma_load_2d(smem_u32(a_smem + (size_t)s * A_TILE_BYTES), &tmA, fb, kb * BK, m0);
                    *(volatile int *)&ctl->issued = it + 1;
                }
                if (stop) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = mbar_wait(smem_u32(&ctl->wfull), 0);
            if (ok) *(volatile int *)&ctl->w_waited = 1;
            int it = 0;
            for (uint32_t i = 0; ok && i < my_tiles; i++) {
                const int buf = (int)(i & 1u);
                const uint32_t use = i >> 1;
                if (*(volatile int *)&ctl->abort) break;
                if (!mbar_wait(smem_u32(&ctl->tempty[buf]), (use & 1u) ^ 1u)) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + (uint32_t)(buf * BN);
                for (int kb = 0; kb < kbs; kb++, it++) {
                    const int s = it % RING;
                    const uint32_t ph = (uint32_t)(it / RING) & 1u;
                    if (!mbar_wait(smem_u32(&ctl->full[s]), ph)) { ok = false; break; }
                    *(volatile int *)&ctl->consumed = it + 1;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t da = umma_desc_sw128(smem_u32(a_smem + (size_t)s * A_TILE_BYTES));
                    const uint64_t db = umma_desc_sw128(smem_u32(w_smem + (size_t)kb * SC::W_KB_BYTES));
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        umma_f16(d, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0);
                    umma_commit(smem_u32(&ctl->empty[s]));
                }
                if (!ok) break;
                umma_commit(smem_u32(&ctl->tfull[buf]));
            }
            if (!ok) {
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                atomicExch(&ctl->abort, 1);
            }
            umma_commit(smem_u32(&ctl->drain));  // arrives once every MMA above retired
        }
    } else {
        // 8 epilogue warps: TMEM lane quarter q = warp % 4, column-chunk parity h
        const int q = warp & 3;
        const int h = (warp - 2) >> 2;
        for (uint32_t i = 0; i < my_tiles; i++) {
            const int buf = (int)(i & 1u);
            const uint32_t use = i >> 1;
            if (!mbar_wait(smem_u32(&ctl->tfull[buf]), use & 1u)) {
                atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                atomicExch(&ctl->abort, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t rowi = (blockIdx.x + i * gridDim.x) * BM + q * 32 + lane;
            const bool valid = rowi < M;
            const uint32_t taddr = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
            if (mode == 2) {
                const uint32_t b = rowi / sp.Q, k2 = rowi - b * sp.Q;
                uint32_t *g = reinterpret_cast<uint32_t *>(out) + (uint64_t)b * sp.Q + k2;
                const uint64_t stride = sp.batch * sp.Q;
                const float2 w = valid ? sp.twiddle[k2] : make_float2(1.f, 0.f);
                for (int c = 32 * h; c < (int)N; c += 64) {
                    uint32_t r[32];
                    tmem_ld32(taddr + (uint32_t)c, r);
                    const uint32_t m1_0 = (uint32_t)c >> 1;
                    if (valid && m1_0 < sp.P)
                        stage1_chunk(r, g, stride, m1_0, sp.P, sp.twiddle[k2 * m1_0], w);
                }
            } else {
                const uint32_t m1 = rowi / (uint32_t)sp.batch, b = rowi - m1 * (uint32_t)sp.batch;
                for (int c = 32 * h; c < (int)N; c += 64) {
                    uint32_t r[32];
                    tmem_ld32(taddr + (uint32_t)c, r);
                    if (!valid) continue;
                    const uint32_t m2_0 = (uint32_t)c >> 1;
                    if (out_dtype == HCT_B200_F16)
                        stage2_chunk<HCT_B200_F16>(r, out, ldo, b, m1, m2_0, sp);
                    else if (out_dtype == HCT_B200_BF16)
                        stage2_chunk<HCT_B200_BF16>(r, out, ldo, b, m1, m2_0, sp);
                    else
                        stage2_chunk<HCT_B200_F32>(r, out, ldo, b, m1, m2_0, sp);
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
        if (!*(volatile int *)&ctl->w_waited && !mbar_wait(smem_u32(&ctl->wfull), 0))
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
    StageParams sp{a.P, a.Q, a.H, 0, a.batch, reinterpret_cast<const float2 *>(a.twiddle), a.scale};
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

template <int BN>
cudaError_t launch_stage(const GemmArgs &a, cudaStream_t s) {
    using SC = StageCfg<BN>;
    if (a.K > (uint64_t)SC::KB_MAX * BK || a.N > (uint64_t)BN) return cudaErrorInvalidValue;
    alignas(64) CUtensorMap ta, tb;
    if (!make_operand_map(&ta, a.A, a.M, a.K, a.lda, BM)) return cudaErrorInvalidValue;
    if (!make_operand_map(&tb, a.B, a.N, a.K, a.ldb, BN)) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(dft_stage_kernel<BN>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SC::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    const uint64_t m_tiles = (a.M + BM - 1) / BM;
    if (m_tiles > 0x7fffffffull) return cudaErrorInvalidValue;
    const uint64_t per_sm = BN == 128 ? 2 : 1;  // shared memory and TMEM allow two 128-wide CTAs
    const uint32_t grid = (uint32_t)std::min<uint64_t>(m_tiles, per_sm * (uint64_t)sm_count());
    StageParams sp{a.P, a.Q, a.H, 0, a.batch, reinterpret_cast<const float2 *>(a.twiddle), a.scale};
    dft_stage_kernel<BN><<<grid, STAGE_THREADS, SC::SMEM_BYTES, s>>>(
        ta, tb, (uint32_t)a.M, (uint32_t)a.N, (uint32_t)a.K, (uint32_t)m_tiles, a.out, a.ldo,
        a.mode, a.out_dtype, a.d_flag, sp);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_umma_gemm(const GemmArgs &a, cudaStream_t s) {
    if (a.M == 0 || a.N == 0) return cudaSuccess;
    if ((a.lda % 8) || (a.ldb % 8) || a.K == 0) return cudaErrorInvalidValue;
    if (a.M > 0x7fffffffull || a.N > 0x7fffffffull || a.K > 0x7fffffffull)
        return cudaErrorInvalidValue;
    if ((a.mode == 2 || a.mode == 3) && (!a.P || !a.Q || !a.batch || a.N > 256 ||
                                         (a.mode == 2 && !a.twiddle)))
        return cudaErrorInvalidValue;
    if (a.mode == 2 || a.mode == 3) {
        if (a.N <= 128 && a.K <= 128) return launch_stage<128>(a, s);
        return launch_stage<256>(a, s);
    }
    if (a.N <= 128) return launch_bn<128>(a, s);
    return launch_bn<256>(a, s);
}

}  // namespace hct
