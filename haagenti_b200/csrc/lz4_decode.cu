// K1: LZ4 block decoder, one warp per independent block.
//
// Restates crates/haagenti-lz4/src/block.rs:261-366 (decompress_block) with
// the same results and the same error variant / position for every input:
//   token -> literal-length extension -> literals -> early exit when
//   output_pos >= output_size -> u16 offset (zero / beyond-output errors)
//   -> match-length extension -> (overlapping) match copy.
// The token stream is inherently serial inside a block, so the warp walks it
// in lock-step (every lane holds the same parse state) and parallelises what
// is wide: 255-run length extensions are scanned 32 bytes at a time with a
// ballot, literal runs and non-overlapping matches are copied as aligned
// 32-bit words (funnel-shifted from an unaligned source), and overlapping
// matches are expanded as out[p + i] = out[p - off + i % off], which only
// reads bytes that were written before the match started.
//
// Every read is checked against the block's compressed length and every
// write against its capacity before it happens: a corrupt block ends with a
// status, never with an out-of-range access or a trap.
//
// Staged variant (container blocks of at most LZ4_STAGE_MAX compressed
// bytes): the warp first pulls its whole compressed block into shared memory
// with 16-byte cp.async copies (the block's bytes all in flight at once, no
// registers held), then parses it and copies its literals from shared
// memory, so the serial token walk costs shared-memory latency instead of
// one DRAM round trip per step.
#include "common.cuh"

namespace hct {
namespace {

constexpr unsigned FULL = 0xffffffffu;

struct ExtResult {
    uint64_t add;   // value added to the length
    uint64_t ip;    // input position after the extension bytes
    bool eof;       // ran out of input before a byte != 255
};

// Length extension (block.rs:277-289 / 328-341): bytes are added while they
// equal 255; the first byte != 255 ends the run (and is added too).
__device__ __forceinline__ ExtResult read_ext(const uint8_t *in, uint64_t in_len, uint64_t ip,
                                              int lane) {
    ExtResult r{0, ip, false};
    for (;;) {
        uint64_t p = r.ip + lane;
        bool valid = p < in_len;
        uint32_t b = valid ? in[p] : 255u;
        unsigned stop = __ballot_sync(FULL, valid && b != 255u);
        if (stop) {
            int first = __ffs(stop) - 1;
            uint32_t last = __shfl_sync(FULL, b, first);
            r.add += 255ull * first + last;
            r.ip += first + 1;
            return r;
        }
        unsigned val = __ballot_sync(FULL, valid);
        if (val != FULL) {  // input ended inside the run: EOF at in_len
            r.eof = true;
            r.ip = in_len;
            return r;
        }
        r.add += 255ull * 32;
        r.ip += 32;
    }
}

// Copy len bytes src -> dst with the warp; [src, src+len) must not overlap
// [dst, dst+len) except that src may precede dst by at least len bytes.
// Destination words are 4-byte aligned; source words are assembled with a
// funnel shift from the two aligned words that hold them.
__device__ __forceinline__ void warp_copy(uint8_t *dst, const uint8_t *src, uint64_t len,
                                          int lane) {
    uint64_t head = (4u - ((uintptr_t)dst & 3u)) & 3u;
    if (head > len) head = len;
    if (lane < (int)head) dst[lane] = src[lane];
    dst += head;
    src += head;
    len -= head;
    const uint64_t nw = len >> 2;
    uint32_t *dw = reinterpret_cast<uint32_t *>(dst);
    const unsigned sh = (unsigned)((uintptr_t)src & 3u);
    const uint32_t *sw = reinterpret_cast<const uint32_t *>((uintptr_t)src & ~(uintptr_t)3);
    if (sh == 0) {
        uint64_t i = lane;
        for (; i + 96 < nw; i += 128) {
            uint32_t a = sw[i], b = sw[i + 32], c = sw[i + 64], d = sw[i + 96];
            dw[i] = a; dw[i + 32] = b; dw[i + 64] = c; dw[i + 96] = d;
        }
        for (; i < nw; i += 32) dw[i] = sw[i];
    } else {
        const unsigned bits = 8u * sh;
        uint64_t i = lane;
        for (; i + 96 < nw; i += 128) {
            uint32_t a0 = sw[i], a1 = sw[i + 1], b0 = sw[i + 32], b1 = sw[i + 33];
            uint32_t c0 = sw[i + 64], c1 = sw[i + 65], d0 = sw[i + 96], d1 = sw[i + 97];
            dw[i] = __funnelshift_r(a0, a1, bits);
            dw[i + 32] = __funnelshift_r(b0, b1, bits);
            dw[i + 64] = __funnelshift_r(c0, c1, bits);
            dw[i + 96] = __funnelshift_r(d0, d1, bits);
        }
        for (; i < nw; i += 32) dw[i] = __funnelshift_r(sw[i], sw[i + 1], bits);
    }
    const uint64_t tail = len & 3u;
    if (lane < (int)tail) dst[nw * 4 + lane] = src[nw * 4 + lane];
}

// staged compressed bytes per warp: the LZ4 bound of a 16 KiB block
// (16384 + 16384 / 255 + 16 = 16464), rounded up
constexpr uint32_t LZ4_STAGE_MAX = 16512;
constexpr uint32_t LZ4_STAGE_BYTES = LZ4_STAGE_MAX + 32;  // + alignment slack
constexpr int LZ4_STAGED_WARPS = 4;                   // warps per CTA of the staged variant

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t sa = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;\n" ::: "memory");
}

// Copies in[0, len) into stage + (in & 15) and returns that pointer: bytes
// up to the first 16-byte boundary and after the last one one by one, the
// aligned body with cp.async (no byte outside [in, in + len) is read).
__device__ __forceinline__ const uint8_t *stage_block(uint8_t *stage, const uint8_t *in,
                                                     uint64_t len, int lane) {
    const uint32_t mis = (uint32_t)((uintptr_t)in & 15u);
    uint8_t *s = stage + mis;
    uint64_t head = (16u - mis) & 15u;
    if (head > len) head = len;
    const uint64_t body_end = head + ((len - head) & ~15ull);
    if ((uint64_t)lane < head) s[lane] = in[lane];
    if ((uint64_t)lane < len - body_end) s[body_end + lane] = in[body_end + lane];
    for (uint64_t j = head + 16ull * lane; j < body_end; j += 512) cp_async16(s + j, in + j);
    cp_async_wait_all();
    __syncwarp();
    return s;
}

template <bool STAGED>
__global__ void __launch_bounds__(256) lz4_decode_blocks_kernel(
    const uint8_t *__restrict__ src, const hct_b200_lz4_block *__restrict__ blocks,
    uint32_t nblocks, uint8_t *dst, hct_b200_status *__restrict__ status) {
    extern __shared__ __align__(16) uint8_t lz4_stage[];
    const int lane = threadIdx.x & 31;
    const uint32_t warps_per_grid = (gridDim.x * blockDim.x) >> 5;
    for (uint32_t bi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; bi < nblocks;
         bi += warps_per_grid) {
        const hct_b200_lz4_block b = blocks[bi];
        const uint8_t *in = src + b.src_off;
        uint8_t *out = dst + b.dst_off;
        const uint64_t in_len = b.src_len, cap = b.dst_cap, osz = b.out_size;
        if (STAGED && in_len <= LZ4_STAGE_MAX) {
            __syncwarp();  // the previous block's reads of the stage are done
            in = stage_block(lz4_stage + (threadIdx.x >> 5) * LZ4_STAGE_BYTES, in, in_len, lane);
        }
        uint64_t ip = 0, op = 0;
        int code = HCT_B200_OK;
        uint64_t epos = 0, eprov = 0;

        while (ip < in_len) {
            const uint32_t token = in[ip];
            ip += 1;
            uint64_t lit = token >> 4;
            uint64_t ml = token & 0x0fu;
            if (lit == 15) {
                ExtResult e = read_ext(in, in_len, ip, lane);
                if (e.eof) { code = HCT_B200_ERR_UNEXPECTED_EOF; epos = e.ip; break; }
                lit += e.add;
                ip = e.ip;
            }
            if (lit > 0) {
                if (ip + lit > in_len) { code = HCT_B200_ERR_UNEXPECTED_EOF; epos = ip; break; }
                if (op + lit > cap) {
                    code = HCT_B200_ERR_BUFFER_TOO_SMALL; epos = op + lit; eprov = cap; break;
                }
                warp_copy(out + op, in + ip, lit, lane);
                ip += lit;
                op += lit;
            }
            if (op >= osz) break;
            if (ip + 2 > in_len) { code = HCT_B200_ERR_UNEXPECTED_EOF; epos = ip; break; }
            const uint64_t offset = (uint64_t)in[ip] | ((uint64_t)in[ip + 1] << 8);
            ip += 2;
            if (offset == 0) { code = HCT_B200_ERR_ZERO_OFFSET; epos = op; break; }
            if (offset > op) { code = HCT_B200_ERR_OFFSET_BEYOND; epos = op; break; }
            ml += 4;
            if ((token & 0x0fu) == 15) {
                ExtResult e = read_ext(in, in_len, ip, lane);
                if (e.eof) { code = HCT_B200_ERR_UNEXPECTED_EOF; epos = e.ip; break; }
                ml += e.add;
                ip = e.ip;
            }
            if (op + ml > cap) {
                code = HCT_B200_ERR_BUFFER_TOO_SMALL; epos = op + ml; eprov = cap; break;
            }
            __syncwarp();  // earlier output visible to every lane
            uint8_t *o = out + op;
            if (offset >= ml) {
                warp_copy(o, o - offset, ml, lane);
            } else {
                const uint8_t *m = o - offset;
                // i % offset advanced incrementally: step 32 mod offset
                const uint32_t off32 = (uint32_t)offset;
                const uint32_t step = 32u % off32;
                uint32_t r = (uint32_t)lane % off32;
                for (uint64_t i = lane; i < ml; i += 32) {
                    o[i] = m[r];
                    r += step;
                    if (r >= off32) r -= off32;
                }
            }
            __syncwarp();
            op += ml;
        }
        if (lane == 0) {
            hct_b200_status s;
            s.code = code;
            s.reserved = 0;
            s.position = code ? epos : 0;
            s.provided = eprov;
            s.written = op;
            status[bi] = s;
        }
        __syncwarp();
    }
}

}  // namespace

cudaError_t launch_lz4_blocks(const uint8_t *d_src, const hct_b200_lz4_block *d_blocks,
                              uint32_t n, uint8_t *d_dst, hct_b200_status *d_status,
                              cudaStream_t s, uint64_t max_src_len) {
    if (n == 0) return cudaSuccess;
    if (max_src_len != 0 && max_src_len <= LZ4_STAGE_MAX) {
        // staged: 4 warps and 64 KiB of shared memory per CTA, 3 CTAs per SM
        const size_t smem = (size_t)LZ4_STAGED_WARPS * LZ4_STAGE_BYTES;
        cudaError_t e = cudaFuncSetAttribute(lz4_decode_blocks_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        uint64_t ctas = (n + LZ4_STAGED_WARPS - 1) / LZ4_STAGED_WARPS;
        if (ctas > 148ull * 3) ctas = 148ull * 3;
        lz4_decode_blocks_kernel<true><<<(unsigned)ctas, 32 * LZ4_STAGED_WARPS, smem, s>>>(
            d_src, d_blocks, n, d_dst, d_status);
        return cudaGetLastError();
    }
    const int threads = 256;  // 8 warps = 8 blocks per CTA
    uint64_t ctas = (n + 7) / 8;
    if (ctas > 148ull * 64) ctas = 148ull * 64;
    lz4_decode_blocks_kernel<false><<<(unsigned)ctas, threads, 0, s>>>(d_src, d_blocks, n, d_dst,
                                                                       d_status);
    return cudaGetLastError();
}

}  // namespace hct
