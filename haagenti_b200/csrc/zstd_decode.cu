// GPU Zstandard decode of a list of jobs (a job: a byte range of the input
// holding one or more concatenated frames, and its output range).  The
// decoder itself is zstd_core.cuh; this file holds the kernels and the
// launch sequence:
//
//   1. zstd_plan_kernel, a thread per job: a job holding one frame of
//      encoder-sized blocks is planned block-parallel and its blocks
//      appended to a descriptor pool;
//   2. zstd_block_kernel, a warp per pooled block: the block's literals
//      straight into the output, with a small workspace (an 11-bit Huffman
//      table) so that 28 warps share an SM;
//   3. zstd_frame_kernel, a warp per job: for a block-parallel job its
//      blocks with sequences (in order; compressed weights have few) and
//      the content checksum; the whole serial decode (every frame form) of
//      any other job and of a block-parallel job that failed, which also
//      reports the error.
//
// Each frame-kernel warp owns a workspace in shared memory (FSE / Huffman
// tables, repeat offsets, a batch of decoded sequences) and 128 KiB of
// literal scratch in device memory.
#include "common.cuh"
#include "zstd_core.cuh"

namespace hct {
namespace {

constexpr int ZWARPS = 4;  // frame kernel: warps (jobs in flight) per CTA
#ifndef ZSTD_MIN_CTAS
#define ZSTD_MIN_CTAS 3  // resident frame-kernel CTAs per SM the register budget allows
#endif
constexpr uint64_t ZSTD_GRID_CAP = 148ull * ZSTD_MIN_CTAS;
constexpr int BWARPS = 4;     // block kernel: warps per CTA
#ifndef ZSTD_BMIN_CTAS
#define ZSTD_BMIN_CTAS 7
#endif
constexpr int BMIN_CTAS = ZSTD_BMIN_CTAS;  // resident block-kernel CTAs per SM
// its Huffman tables: zstd's encoders write literal tables of at most 11
// bits (a block with a 12-bit table fails here and its frame is decoded
// serially); the smaller workspace lets 7 CTAs share an SM
typedef zs::HufWsT<11> BlockWs;
constexpr uint32_t PLAN_THREADS = 128;

// Scratch layout: frame-kernel literal scratch, then the job plans, the
// pool and slot counters, the block descriptor pool and the literal slots
// of blocks with sequences.
constexpr uint32_t SEQ_SLOTS = 128;
struct ScratchLayout {
    size_t lit, plans, counter, pool, slots, total;
    uint32_t pool_cap;
};

ScratchLayout scratch_layout(uint32_t n) {
    ScratchLayout L;
    const uint64_t ctas = ((uint64_t)n + ZWARPS - 1) / ZWARPS;
    const uint64_t grid = ctas < ZSTD_GRID_CAP ? (ctas ? ctas : 1) : ZSTD_GRID_CAP;
    L.lit = 0;
    L.plans = grid * ZWARPS * zs::LIT_SCRATCH;
    L.counter = L.plans + (((size_t)n * sizeof(zs::JobPlan) + 255) & ~(size_t)255);
    L.pool = L.counter + 256;
    L.pool_cap = 4 * n + 16384;  // blocks; a job that does not fit is decoded serially
    L.slots = L.pool + (((size_t)L.pool_cap * sizeof(zs::BlockDesc) + 255) & ~(size_t)255);
    L.total = L.slots + (size_t)SEQ_SLOTS * zs::LIT_SCRATCH;
    return L;
}

__global__ void __launch_bounds__(PLAN_THREADS) zstd_plan_kernel(
    const uint8_t *__restrict__ src, const hct_b200_zstd_job *__restrict__ jobs, uint32_t n,
    zs::JobPlan *__restrict__ plans, zs::BlockDesc *__restrict__ pool, uint32_t *pool_used,
    uint32_t pool_cap) {
    const uint32_t j = blockIdx.x * PLAN_THREADS + threadIdx.x;
    if (j >= n) return;
    const hct_b200_zstd_job jd = jobs[j];
    zs::JobPlan jp{0, ~0ull, 0, 0, 0, 0, 0, 0, 0};
    uint32_t cnt = 0;
    bool par = zs::plan_job(src + jd.src_off, jd.src_len, jd.dst_cap, j, &jp, nullptr, &cnt);
    if (par) {
        const uint32_t base = atomicAdd(pool_used, cnt);
        if ((uint64_t)base + cnt <= pool_cap) {
            zs::plan_job(src + jd.src_off, jd.src_len, jd.dst_cap, j, &jp, pool + base, &cnt);
            jp.base = base;
            // literal slots for the blocks with sequences, while they last
            for (uint32_t i = 0; i < cnt && jp.nseq; i++) {
                if (!(pool[base + i].meta & zs::META_SEQ)) continue;
                const uint32_t sl = atomicAdd(pool_used + 1, 1u);
                pool[base + i].slot = sl < SEQ_SLOTS ? sl : ~0u;
            }
        } else {
            par = false;  // pool full: mark the reserved slots empty
            for (uint64_t i = base; i < pool_cap && i < (uint64_t)base + cnt; i++)
                pool[i].meta = 3u << 18;
        }
    }
    jp.mode = par ? 1 : 0;
    plans[j] = jp;
}

__global__ void __launch_bounds__(BWARPS * 32, BMIN_CTAS) zstd_block_kernel(
    const uint8_t *__restrict__ src, const hct_b200_zstd_job *__restrict__ jobs,
    zs::JobPlan *plans, const zs::BlockDesc *__restrict__ pool, const uint32_t *pool_used,
    uint32_t pool_cap, uint8_t *dst, uint8_t *slots) {
    __shared__ BlockWs hws[BWARPS];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    BlockWs *ws = hws + warp;
    const uint32_t used0 = *pool_used;
    const uint32_t used = used0 < pool_cap ? used0 : pool_cap;
    const uint32_t nw = gridDim.x * BWARPS;
    for (uint32_t i = blockIdx.x * BWARPS + warp; i < used; i += nw) {
        zs::BlockDesc e = pool[i];
        if (((e.meta >> 18) & 3) == 3) continue;
        const hct_b200_zstd_job jd = jobs[e.job];
        uint8_t *out = dst + jd.dst_off;
        if (e.meta & zs::META_SEQ) {
            // a block with sequences (the frame kernel's): its Huffman
            // literals into its slot
            if (e.slot == ~0u || (src[jd.src_off + e.src] & 3) < 2) continue;
            out = slots + (uint64_t)e.slot * zs::LIT_SCRATCH;
            e.out = 0;
        }
        const bool ok = zs::decode_block(ws, src + jd.src_off, e, out, lane, 32);
        if (!ok && lane == 0) plans[e.job].fail = 1;
        __syncwarp();
    }
}

__global__ void __launch_bounds__(ZWARPS * 32, ZSTD_MIN_CTAS) zstd_frame_kernel(
    const uint8_t *__restrict__ src, const hct_b200_zstd_job *__restrict__ jobs, uint32_t n,
    const zs::JobPlan *__restrict__ plans, const zs::BlockDesc *__restrict__ pool,
    const uint8_t *slots, uint8_t *dst, hct_b200_status *__restrict__ status, uint8_t *scratch) {
    extern __shared__ uint8_t zsm[];
    __shared__ uint64_t acc[ZWARPS][4];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    zs::Workspace *ws = reinterpret_cast<zs::Workspace *>(zsm) + warp;
    const uint64_t gw = (uint64_t)blockIdx.x * ZWARPS + warp;
    const uint64_t nw = (uint64_t)gridDim.x * ZWARPS;
    uint8_t *lit = scratch + gw * zs::LIT_SCRATCH;
    for (uint64_t j = gw; j < n; j += nw) {
        const hct_b200_zstd_job jd = jobs[j];
        const zs::JobPlan jp = plans[j];
        const zs::Job job{src + jd.src_off, jd.src_len, dst + jd.dst_off, jd.dst_cap, lit};
        zs::Result r;
        bool par = jp.mode == 1 && jp.fail == 0;
        // block-parallel job: the blocks with sequences, then the checksum
        if (par && jp.nseq) par = zs::decode_seq_blocks(ws, job, jp, pool + jp.base, slots, lane, 32);
        if (par) {
            r = zs::Result{zs::OK, jp.lastpos, jp.total};
            if (jp.ckpos != ~0ull) {
                const uint64_t h = zs::xxh64(dst + jd.dst_off, jp.total, lane, 32, acc[warp],
                                             reinterpret_cast<uint64_t *>(ws->huf));
                if ((uint32_t)h != zs::rd32(src + jd.src_off + jp.ckpos)) {
                    r.code = zs::E_CHECKSUM;
                    r.pos = jp.ckpos;
                }
            }
        } else {
            r = zs::decode(ws, job, lane, 32, acc[warp]);
        }
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

size_t zstd_scratch_bytes(uint32_t n) { return scratch_layout(n).total; }

cudaError_t launch_zstd_decode(const uint8_t *d_src, const hct_b200_zstd_job *d_jobs, uint32_t n,
                               uint8_t *d_dst, hct_b200_status *d_status, uint8_t *d_scratch,
                               cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const ScratchLayout L = scratch_layout(n);
    zs::JobPlan *plans = reinterpret_cast<zs::JobPlan *>(d_scratch + L.plans);
    uint32_t *counter = reinterpret_cast<uint32_t *>(d_scratch + L.counter);
    zs::BlockDesc *pool = reinterpret_cast<zs::BlockDesc *>(d_scratch + L.pool);
    uint8_t *slots = d_scratch + L.slots;
    cudaError_t e = cudaMemsetAsync(counter, 0, 2 * sizeof(uint32_t), s);  // pool, slots
    if (e != cudaSuccess) return e;
    zstd_plan_kernel<<<(n + PLAN_THREADS - 1) / PLAN_THREADS, PLAN_THREADS, 0, s>>>(
        d_src, d_jobs, n, plans, pool, counter, L.pool_cap);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // persistent: every warp loops over the pooled blocks
    zstd_block_kernel<<<148 * BMIN_CTAS, BWARPS * 32, 0, s>>>(d_src, d_jobs, plans, pool, counter,
                                                               L.pool_cap, d_dst, slots);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const size_t smem = sizeof(zs::Workspace) * ZWARPS;
    e = cudaFuncSetAttribute(zstd_frame_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    // as many CTAs as the literal scratch provides for
    const uint64_t ctas = ((uint64_t)n + ZWARPS - 1) / ZWARPS;
    const uint64_t grid = ctas < ZSTD_GRID_CAP ? ctas : ZSTD_GRID_CAP;
    zstd_frame_kernel<<<(unsigned)grid, ZWARPS * 32, smem, s>>>(d_src, d_jobs, n, plans, pool, slots,
                                                                d_dst, d_status, d_scratch + L.lit);
    return cudaGetLastError();
}

}  // namespace hct
