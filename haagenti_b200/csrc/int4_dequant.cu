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

#include <algorithm>
#include <cuda_fp16.h>

#include "common.cuh"

#ifndef DQ_TILE_ELEMS
#define DQ_TILE_ELEMS 16384
#endif

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

// ---- dequant_int4: 16 KiB-element tiles staged by cp.async.bulk ----------
//
// A launch dequantises a batch of tensors ("jobs").  Each job is cut into
// tiles of DQ_TILE elements; CTAs take tiles t = blockIdx.x + i * gridDim.x
// over the whole batch.  A tile's 8 KiB of nibbles and 1 KiB of f16 scales
// are copied into shared memory by two 1-D bulk copies (cp.async.bulk, no
// multicast) issued by thread 0 up to DQ_STAGES tiles ahead and completed
// on an mbarrier; a job whose nibble section is not 16-byte aligned, and the
// last partial tile of every job, are read from global memory directly.
// Within a tile, warp w takes elements [2048 w, 2048 w + 2048); lane l of
// step j takes the 8 elements at 2048 w + 256 j + 8 l (one nibble word, one
// scale), so every store instruction of a warp writes 1 KiB (f32) or 512 B
// (f16/bf16) of contiguous output with 32- or 16-byte stores.
constexpr int DQ_THREADS = 256;
constexpr int DQ_TILE = DQ_TILE_ELEMS;
constexpr int DQ_STEPS = DQ_TILE / 2048;  // 8-element steps per lane within a tile
constexpr int DQ_WARP_SPAN = 256 * DQ_STEPS;  // elements per warp per tile
constexpr int DQ_NIB = DQ_TILE / 2;   // nibble bytes per tile
constexpr int DQ_SC = DQ_TILE / 16;   // scale bytes per tile (f16 per 32 elements)
constexpr int DQ_STAGES = 3;
constexpr int DQ_STAGE_BYTES = DQ_NIB + DQ_SC;
constexpr uint64_t DQ_WAIT_NS = 2000000000ull;

struct DqJob {
    const uint8_t *data;  // f16 scales at data, nibbles at data + sb
    void *out;
    uint64_t sb;          // 2 * ceil(num_elements / 32)
    uint64_t n;           // elements written
    uint64_t tile0;       // first tile of the job within the launch
    uint64_t bulk_tiles;  // leading whole tiles staged by the bulk copies
    uint32_t vec;         // out is aligned for 32-byte (f32) / 16-byte (f16, bf16) stores
    uint32_t pad;
};
struct DqBatch {
    DqJob job[DQ_MAX_JOBS];
    uint32_t njobs;
    uint64_t total_tiles;
};

__device__ __forceinline__ uint32_t dq_smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ bool dq_try_wait(uint32_t bar, uint32_t parity) {
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

// Bounded wait on an mbarrier phase (iteration count and %globaltimer).
__device__ __forceinline__ bool dq_wait(uint32_t bar, uint32_t parity) {
    if (dq_try_wait(bar, parity)) return true;
    uint64_t t0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    for (uint32_t i = 1; i < (1u << 30); ++i) {
        if (dq_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            uint64_t t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            if (t - t0 > DQ_WAIT_NS) return false;
        }
    }
    return false;
}

__device__ __forceinline__ uint32_t dq_job_of(const DqBatch &b, uint64_t t) {
    uint32_t lo = 0, hi = b.njobs - 1;
    while (lo < hi) {  // last job whose tile0 <= t
        const uint32_t mid = (lo + hi + 1) / 2;
        if (b.job[mid].tile0 <= t) lo = mid;
        else hi = mid - 1;
    }
    return lo;
}

// thread 0: the two bulk copies of tile `local` of job j into stage `slot`
__device__ __forceinline__ void dq_issue(const DqJob &jb, uint64_t local, uint8_t *stage,
                                         uint32_t bar) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"((uint32_t)DQ_STAGE_BYTES)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dq_smem_u32(stage)),
        "l"(jb.data + jb.sb + local * DQ_NIB), "r"((uint32_t)DQ_NIB), "r"(bar)
        : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dq_smem_u32(stage + DQ_NIB)),
        "l"(jb.data + local * DQ_SC), "r"((uint32_t)DQ_SC), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void st_v8_f32(float *p, const float (&v)[8]) {
    asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]),
                 "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
                 : "memory");
}

// 8 elements from one nibble word (low nibble first) and their f32 scale:
// (nibble - 8) as an exact float is (2^23 + nibble) - (2^23 + 8).
template <int DT>
__device__ __forceinline__ void dq_store1(void *out, uint64_t e, float v) {
    if (DT == HCT_B200_F32) reinterpret_cast<float *>(out)[e] = v;
    else if (DT == HCT_B200_F16) reinterpret_cast<uint16_t *>(out)[e] = to_f16(v);
    else reinterpret_cast<uint16_t *>(out)[e] = to_bf16(v);
}

template <int DT>
__device__ __forceinline__ void dq_emit8(void *out, uint64_t e, uint32_t w, float scale,
                                         bool vec) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; k++)
        v[k] = __fmul_rn(__int_as_float(0x4B000000 | ((w >> (4 * k)) & 0xfu)) - 8388616.0f, scale);
    if (!vec) {
#pragma unroll
        for (int k = 0; k < 8; k++) dq_store1<DT>(out, e + k, v[k]);
    } else if (DT == HCT_B200_F32) {
        st_v8_f32(reinterpret_cast<float *>(out) + e, v);
    } else {
        uint32_t h[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t a = DT == HCT_B200_F16 ? to_f16(v[2 * k]) : to_bf16(v[2 * k]);
            const uint32_t c = DT == HCT_B200_F16 ? to_f16(v[2 * k + 1]) : to_bf16(v[2 * k + 1]);
            h[k] = a | (c << 16);
        }
        *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(out) + e) =
            make_uint4(h[0], h[1], h[2], h[3]);
    }
}

template <int DT>
__global__ void __launch_bounds__(DQ_THREADS) dequant_int4_tiles_kernel(
    const __grid_constant__ DqBatch b, int *flag) {
    extern __shared__ __align__(128) uint8_t dq_smem[];
    __shared__ __align__(8) uint64_t bar[DQ_STAGES];
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < DQ_STAGES; s++)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(dq_smem_u32(&bar[s]))
                         : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    const uint64_t T = b.total_tiles;
    auto bulk_at = [&](uint64_t i, uint32_t *jo, uint64_t *lo) -> bool {
        const uint64_t t = blockIdx.x + i * gridDim.x;
        if (t >= T) return false;
        const uint32_t j = dq_job_of(b, t);
        *jo = j;
        *lo = t - b.job[j].tile0;
        return *lo < b.job[j].bulk_tiles;
    };
    // armed[s]: a copy into stage s is in flight (thread 0's view)
    uint32_t armed = 0, phase = 0;
    if (tid == 0) {
        for (int i = 0; i < DQ_STAGES; i++) {
            uint32_t j;
            uint64_t lo;
            if (bulk_at(i, &j, &lo)) {
                dq_issue(b.job[j], lo, dq_smem + i * DQ_STAGE_BYTES, dq_smem_u32(&bar[i]));
                armed |= 1u << i;
            }
        }
    }
    bool aborted = false;
    for (uint64_t i = 0;; i++) {
        const uint64_t t = blockIdx.x + i * gridDim.x;
        if (t >= T) break;
        const uint32_t j = dq_job_of(b, t);
        const DqJob &jb = b.job[j];
        const uint64_t local = t - jb.tile0;
        const uint64_t e0 = local * DQ_TILE;  // first element of the tile within the job
        const int slot = (int)(i % DQ_STAGES);
        if (local < jb.bulk_tiles) {
            const bool ok = dq_wait(dq_smem_u32(&bar[slot]), (phase >> slot) & 1u);
            if (__syncthreads_or(!ok)) {
                if (tid == 0 && flag) atomicExch(flag, HCT_B200_ERR_TIMEOUT);
                aborted = true;
                break;
            }
            phase ^= 1u << slot;
            const uint8_t *st = dq_smem + slot * DQ_STAGE_BYTES;
            uint32_t w[DQ_STEPS];
            float sc[DQ_STEPS];
#pragma unroll
            for (int k = 0; k < DQ_STEPS; k++) {
                const uint32_t wi = (DQ_WARP_SPAN / 8) * warp + 32 * k + lane;  // nibble word
                w[k] = reinterpret_cast<const uint32_t *>(st)[wi];
                sc[k] = f16_bits_to_f32(
                    reinterpret_cast<const uint16_t *>(st + DQ_NIB)[wi >> 2]);
            }
            __syncthreads();  // stage consumed: refill it
            if (tid == 0) {
                armed &= ~(1u << slot);
                uint32_t jn;
                uint64_t ln;
                if (bulk_at(i + DQ_STAGES, &jn, &ln)) {
                    dq_issue(b.job[jn], ln, dq_smem + slot * DQ_STAGE_BYTES,
                             dq_smem_u32(&bar[slot]));
                    armed |= 1u << slot;
                }
            }
#pragma unroll
            for (int k = 0; k < DQ_STEPS; k++)
                dq_emit8<DT>(jb.out, e0 + DQ_WARP_SPAN * warp + 256 * k + 8 * lane, w[k], sc[k],
                             true);
        } else {
            // direct loads: a misaligned job, or the job's last (partial) tile
            const uint8_t *nib = jb.data + jb.sb;
#pragma unroll 2
            for (int k = 0; k < DQ_STEPS; k++) {
                const uint64_t e = e0 + DQ_WARP_SPAN * warp + 256 * k + 8 * lane;
                if (e >= jb.n) continue;
                const uint64_t blk = e >> 5;
                const float scale = f16_bits_to_f32((uint32_t)jb.data[2 * blk] |
                                                    ((uint32_t)jb.data[2 * blk + 1] << 8));
                if (e + 8 <= jb.n) {
                    dq_emit8<DT>(jb.out, e, ld_u32_any(nib + (e >> 1)), scale, jb.vec != 0);
                } else {
                    for (uint64_t x = e; x < jb.n; x++) {
                        const uint32_t byte = nib[x >> 1];
                        const uint32_t nb = (x & 1) ? byte >> 4 : byte & 0xfu;
                        dq_store1<DT>(jb.out, x, deq(nb, scale));
                    }
                }
            }
        }
    }
    // teardown: copies still in flight into this CTA's stages (abort path only)
    if (aborted && tid == 0) {
        for (int s = 0; s < DQ_STAGES; s++)
            if (armed & (1u << s)) {
                if (!dq_wait(dq_smem_u32(&bar[s]), (phase >> s) & 1u) && flag)
                    atomicExch(flag, HCT_B200_ERR_TIMEOUT);
            }
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

namespace {

int dq_max_grid() {
    static int g = 0;
    if (!g) {
        int dev = 0, sms = 148, per = 0;
        if (cudaGetDevice(&dev) == cudaSuccess)
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const size_t smem = (size_t)DQ_STAGES * DQ_STAGE_BYTES;
        if (cudaFuncSetAttribute(dequant_int4_tiles_kernel<HCT_B200_F32>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
            cudaFuncSetAttribute(dequant_int4_tiles_kernel<HCT_B200_F16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
            cudaFuncSetAttribute(dequant_int4_tiles_kernel<HCT_B200_BF16>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &per, dequant_int4_tiles_kernel<HCT_B200_F32>, DQ_THREADS, smem) ||
            per < 1)
            per = 4;
        g = sms * per;
    }
    return g;
}

}  // namespace

cudaError_t launch_dequant_int4_batch(const Int4Job *jobs, uint32_t njobs, int dtype, int *d_flag,
                                      cudaStream_t s) {
    const size_t esz = dtype == HCT_B200_F32 ? 4 : 2;
    for (uint32_t j0 = 0; j0 < njobs; j0 += DQ_MAX_JOBS) {
        DqBatch b{};
        uint64_t tiles = 0;
        for (uint32_t j = j0; j < njobs && b.njobs < DQ_MAX_JOBS; j++) {
            const Int4Job &in = jobs[j];
            if (in.n_written == 0) continue;
            if ((uintptr_t)in.out % esz) return cudaErrorInvalidValue;
            DqJob &d = b.job[b.njobs++];
            d.data = in.data;
            d.out = in.out;
            d.sb = (in.num_elements + 31) / 32 * 2;
            d.n = in.n_written;
            d.tile0 = tiles;
            d.vec = (uintptr_t)in.out % (dtype == HCT_B200_F32 ? 32 : 16) == 0;
            const bool aligned = ((uintptr_t)in.data % 16 == 0) && (d.sb % 16 == 0) && d.vec;
            d.bulk_tiles = aligned ? in.n_written / DQ_TILE : 0;
            tiles += (in.n_written + DQ_TILE - 1) / DQ_TILE;
        }
        if (!b.njobs) continue;
        b.total_tiles = tiles;
        const unsigned grid = (unsigned)std::min<uint64_t>(tiles, (uint64_t)dq_max_grid());
        const size_t smem = (size_t)DQ_STAGES * DQ_STAGE_BYTES;
        switch (dtype) {
            case HCT_B200_F32:
                dequant_int4_tiles_kernel<HCT_B200_F32><<<grid, DQ_THREADS, smem, s>>>(b, d_flag);
                break;
            case HCT_B200_F16:
                dequant_int4_tiles_kernel<HCT_B200_F16><<<grid, DQ_THREADS, smem, s>>>(b, d_flag);
                break;
            default:
                dequant_int4_tiles_kernel<HCT_B200_BF16><<<grid, DQ_THREADS, smem, s>>>(b, d_flag);
                break;
        }
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_dequant_int4(const uint8_t *d_data, size_t data_len, size_t n_written,
                                size_t num_elements, void *d_out, int dtype, int *d_flag,
                                cudaStream_t s) {
    (void)data_len;
    if (n_written == 0) return cudaSuccess;
    Int4Job j{d_data, d_out, num_elements, n_written};
    return launch_dequant_int4_batch(&j, 1, dtype, d_flag, s);
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
