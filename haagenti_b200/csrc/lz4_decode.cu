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
// matches (out[p] = out[p - off]) are expanded from the period held in
// registers when off <= 32, else by copying the first period and doubling
// the copied prefix; no copy reads a byte that it writes.
//
// Every read is checked against the block's compressed length and every
// write against its capacity before it happens: a corrupt block ends with a
// status, never with an out-of-range access or a trap.
//
// Staged variant (container blocks: at most LZ4_STAGE_MAX compressed and
// LZ4_OUT_MAX decompressed bytes): the warp first pulls its whole compressed
// block into shared memory with 16-byte cp.async copies (all of its bytes in
// flight at once, no registers held), decodes it into a shared-memory output
// buffer -- token walk, literal copies and match sources all at
// shared-memory latency, and the warp barriers between steps drain no
// global stores -- and finally writes the block out with 16-byte stores.
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

// 16 source bytes starting K words + sh bits into the aligned 32 bytes at q
// (two 16-byte loads; both granules hold a byte of the 16 wanted when the
// start is not 16-byte aligned, which is the only case that calls this).
template <int K>
__device__ __forceinline__ uint4 src16(const uint4 *q, uint32_t sh) {
    const uint4 a = q[0], b = q[1];
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    return make_uint4(__funnelshift_r(w[K], w[K + 1], sh), __funnelshift_r(w[K + 1], w[K + 2], sh),
                      __funnelshift_r(w[K + 2], w[K + 3], sh), __funnelshift_r(w[K + 3], w[K + 4], sh));
}

// nch 16-byte chunks to the aligned d1 from s1 ((s1 & 15) = 4 K + sh / 8, not 0),
// 4 chunks in flight per lane
template <int K>
__device__ __forceinline__ void wide_chunks(uint4 *d1, const uint8_t *s1, uint64_t nch, int lane) {
    const uint4 *q = reinterpret_cast<const uint4 *>((uintptr_t)s1 & ~(uintptr_t)15);
    const uint32_t sh = (uint32_t)((uintptr_t)s1 & 3u) * 8u;
    uint64_t c = (uint64_t)lane;
    for (; c + 96 < nch; c += 128) {
        const uint4 v0 = src16<K>(q + c, sh), v1 = src16<K>(q + c + 32, sh);
        const uint4 v2 = src16<K>(q + c + 64, sh), v3 = src16<K>(q + c + 96, sh);
        d1[c] = v0;
        d1[c + 32] = v1;
        d1[c + 64] = v2;
        d1[c + 96] = v3;
    }
    for (; c < nch; c += 32) d1[c] = src16<K>(q + c, sh);
}

// Literal copy in device memory (no overlap): bytes up to a 16-byte aligned
// destination, then 16-byte stores with 4 chunks in flight per lane (2 KiB
// per warp: the copy of an incompressible block is latency-bound
// otherwise), then the tail.  An aligned source moves with one 16-byte load
// per chunk; otherwise each chunk is cut from two aligned 16-byte loads, the
// word offset (the same for the whole run) a compile-time case.  No load
// reads a 16-byte granule without a byte of [src, src + len).
__device__ __forceinline__ void warp_copy_wide(uint8_t *dst, const uint8_t *src, uint64_t len,
                                               int lane) {
    uint64_t head = (16u - ((uintptr_t)dst & 15u)) & 15u;
    if (head > len) head = len;
    if ((uint64_t)lane < head) dst[lane] = src[lane];
    const uint64_t nch = (len - head) >> 4;
    if (nch) {
        const uint8_t *s1 = src + head;
        uint4 *d1 = reinterpret_cast<uint4 *>(dst + head);
        const uint32_t o = (uint32_t)((uintptr_t)s1 & 15u);
        if (o == 0) {
            const uint4 *q = reinterpret_cast<const uint4 *>(s1);
            uint64_t c = (uint64_t)lane;
            for (; c + 96 < nch; c += 128) {
                const uint4 v0 = q[c], v1 = q[c + 32], v2 = q[c + 64], v3 = q[c + 96];
                d1[c] = v0;
                d1[c + 32] = v1;
                d1[c + 64] = v2;
                d1[c + 96] = v3;
            }
            for (; c < nch; c += 32) d1[c] = q[c];
        } else {
            switch (o >> 2) {  // uniform across the warp
                case 0: wide_chunks<0>(d1, s1, nch, lane); break;
                case 1: wide_chunks<1>(d1, s1, nch, lane); break;
                case 2: wide_chunks<2>(d1, s1, nch, lane); break;
                default: wide_chunks<3>(d1, s1, nch, lane); break;
            }
        }
    }
    const uint64_t t0 = head + 16 * nch;
    if ((uint64_t)lane < len - t0) dst[t0 + lane] = src[t0 + lane];
}

// staged compressed bytes per warp: the LZ4 bound of a 16 KiB block
// (16384 + 16384 / 255 + 16 = 16464), rounded up
constexpr uint32_t LZ4_STAGE_MAX = 16512;
constexpr uint32_t LZ4_STAGE_BYTES = LZ4_STAGE_MAX + 32;  // + alignment slack
constexpr uint32_t LZ4_OUT_MAX = 16384;                  // staged decompressed bytes per warp
constexpr uint32_t LZ4_OUT_BYTES = LZ4_OUT_MAX + 32;
constexpr uint32_t LZ4_SLOT_BYTES = LZ4_STAGE_BYTES + LZ4_OUT_BYTES;
constexpr int LZ4_STAGED_WARPS = 2;  // warps per CTA: 64 KiB of shared memory, 3 CTAs per SM
#ifndef LZ4_STAGED_MAX_CTAS
#define LZ4_STAGED_MAX_CTAS (148ull * 3)  // grid cap: one resident wave, CTAs loop over blocks
#endif

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

// Overlapping match with period off <= 32: o[p] = o[p - off] for p < ml.
// Lane r holds the period's byte r (read once, written before the match);
// every output byte is a shuffle of it, stored 4 bytes per lane from the
// first 4-byte boundary, so the expansion reads no memory it writes.
__device__ __forceinline__ void expand_short_period(uint8_t *o, uint32_t off, uint64_t ml,
                                                    int lane) {
    const uint32_t pv = (uint32_t)lane < off ? (uint32_t)o[(int64_t)lane - (int64_t)off] : 0u;
    uint64_t head = (4u - ((uintptr_t)o & 3u)) & 3u;
    if (head > ml) head = ml;
    const uint32_t hb = __shfl_sync(FULL, pv, (uint32_t)lane % off);
    if ((uint64_t)lane < head) o[lane] = (uint8_t)hb;
    const uint64_t nw = (ml - head) >> 2;
    uint32_t *dw = reinterpret_cast<uint32_t *>(o + head);
    uint32_t r = (uint32_t)((head + 4ull * (uint32_t)lane) % off);  // period index of my word
    const uint32_t step = 128u % off;                                 // 32 words per iteration
    for (uint64_t j0 = 0; j0 < nw; j0 += 32) {
        const uint32_t r1 = r + 1 == off ? 0u : r + 1;
        const uint32_t r2 = r1 + 1 == off ? 0u : r1 + 1;
        const uint32_t r3 = r2 + 1 == off ? 0u : r2 + 1;
        const uint32_t b0 = __shfl_sync(FULL, pv, r);
        const uint32_t b1 = __shfl_sync(FULL, pv, r1);
        const uint32_t b2 = __shfl_sync(FULL, pv, r2);
        const uint32_t b3 = __shfl_sync(FULL, pv, r3);
        if (j0 + lane < nw) dw[j0 + lane] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        r += step;
        if (r >= off) r -= off;
    }
    const uint64_t t0 = head + 4 * nw;  // fewer than 4 bytes remain
    const uint32_t tb = __shfl_sync(FULL, pv, (uint32_t)((t0 + (uint32_t)lane) % off));
    if ((uint64_t)lane < ml - t0) o[t0 + lane] = (uint8_t)tb;
}

// Writes the staged output sout[0, n) to gdst[0, n); sout and gdst agree
// modulo 16, so the body moves as aligned 16-byte words.
__device__ __forceinline__ void store_block(uint8_t *gdst, const uint8_t *sout, uint64_t n,
                                            int lane) {
    uint64_t head = (16u - ((uintptr_t)gdst & 15u)) & 15u;
    if (head > n) head = n;
    const uint64_t body_end = head + ((n - head) & ~15ull);
    if ((uint64_t)lane < head) gdst[lane] = sout[lane];
    if ((uint64_t)lane < n - body_end) gdst[body_end + lane] = sout[body_end + lane];
    for (uint64_t j = head + 16ull * lane; j < body_end; j += 512)
        *reinterpret_cast<uint4 *>(gdst + j) = *reinterpret_cast<const uint4 *>(sout + j);
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
        uint8_t *const gout = out;
        const bool staged = STAGED && in_len <= LZ4_STAGE_MAX && cap <= LZ4_OUT_MAX;
        if (staged) {
            uint8_t *slot = lz4_stage + (threadIdx.x >> 5) * LZ4_SLOT_BYTES;
            __syncwarp();  // the previous block's reads of the slot are done
            in = stage_block(slot, in, in_len, lane);
            out = slot + LZ4_STAGE_BYTES + ((uintptr_t)gout & 15u);
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
                if (lit <= 32) {  // short run: one byte per lane
                    if ((uint64_t)lane < lit) out[op + lane] = in[ip + lane];
                } else if (!staged && lit >= 1024) {
                    // the bytes after the run (offset, next token, its length
                    // bytes, the next short sequences) are the next reads of the
                    // serial walk: ask for their 4 lines while the run is copied
                    if (lane < 4 && ip + lit + 128ull * lane < in_len)
                        asm volatile("prefetch.global.L1 [%0];" ::"l"(in + ip + lit + 128ull * lane));
                    warp_copy_wide(out + op, in + ip, lit, lane);
                } else {
                    warp_copy(out + op, in + ip, lit, lane);
                }
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
            if (offset >= ml && ml <= 32) {  // short, non-overlapping: one byte per lane
                if ((uint64_t)lane < ml) o[lane] = o[(int64_t)lane - (int64_t)offset];
            } else if (offset >= ml) {
                warp_copy(o, o - offset, ml, lane);
            } else if (offset <= 32) {
                expand_short_period(o, (uint32_t)offset, ml, lane);
            } else {
                // the match is periodic with period offset: copy the first
                // period (it only reads bytes before o), then double the
                // copied prefix; every copy reads bytes written before it
                warp_copy(o, o - offset, offset, lane);
                uint64_t done = offset;
                while (done < ml) {
                    __syncwarp();
                    const uint64_t n = done < ml - done ? done : ml - done;
                    warp_copy(o + done, o, n, lane);
                    done += n;
                }
            }
            __syncwarp();
            op += ml;
        }
        if (staged) {
            __syncwarp();
            store_block(gout, out, op, lane);
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
        // staged: 2 warps and 64 KiB of shared memory per CTA, 3 CTAs per SM
        const size_t smem = (size_t)LZ4_STAGED_WARPS * LZ4_SLOT_BYTES;
        cudaError_t e = cudaFuncSetAttribute(lz4_decode_blocks_kernel<true>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        uint64_t ctas = (n + LZ4_STAGED_WARPS - 1) / LZ4_STAGED_WARPS;
        if (ctas > LZ4_STAGED_MAX_CTAS) ctas = LZ4_STAGED_MAX_CTAS;
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
