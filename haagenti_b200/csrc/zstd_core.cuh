// Zstandard frame decoder (RFC 8878), written for one warp per job.
//
// The reference decodes zstd data through the `zstd` crate (libzstd):
// HoloTensorReader::read_fragment for fragments whose index entry has flag
// bit 0 (crates/haagenti-hct/src/holotensor.rs:2081-2091) and
// GpuDecompressor::try_zstd_decompress for zstd-wrapped HCT data
// (crates/haagenti-cuda/src/decompress.rs:296-319), both `zstd::decode_all`:
// every frame of the input in turn (skippable frames skipped), the frames'
// contents concatenated.  This decoder follows the format as RFC 8878
// specifies it and reports an error wherever libzstd's decoder does for the
// checks listed at the functions below.
//
// Work split inside a warp (nl lanes; the same code runs with nl = 1 on the
// host):
//   * frame, block and section headers: every lane parses them (the same
//     bytes, so the lanes agree without communication);
//   * FSE tables, Huffman weights and the sequence bitstream: lane 0,
//     results in the warp's workspace; the Huffman decoding table is then
//     filled by all lanes;
//   * the 4 Huffman literal streams: one lane each;
//   * raw / RLE blocks, literal copies and match copies: all lanes (a match
//     with offset < length repeats the period-`offset` pattern, so each output
//     byte is read from the bytes before the match and no lane waits on
//     another within a copy);
//   * XXH64 content checksum: lanes 0-3 run the 4 accumulators.
// A frame whose blocks regenerate the encoder's block size is also decoded
// block by block in parallel (plan_job, decode_block, decode_seq_blocks at
// the end of this file; the kernels are in zstd_decode.cu).
#pragma once

#include <cstddef>
#include <cstdint>

#if defined(__CUDACC__)
#define ZHD __host__ __device__ __forceinline__
// rarely run parts (table construction, block headers) stay out of line so
// their registers are not live across the hot loops
#define ZCOLD __host__ __device__ __noinline__
#else
#define ZHD inline
#define ZCOLD inline
#endif

#if defined(__CUDA_ARCH__)
#define ZUNROLL _Pragma("unroll")
#else
#define ZUNROLL
#endif

namespace hct {
namespace zs {

#if defined(__CUDA_ARCH__)
__device__ __forceinline__ void warp_sync() { __syncwarp(); }
__device__ __forceinline__ uint32_t warp_min(uint32_t v) { return __reduce_min_sync(0xffffffffu, v); }
__device__ __forceinline__ uint64_t bcast0(uint64_t v) { return __shfl_sync(0xffffffffu, v, 0); }
#else
inline uint64_t bcast0(uint64_t v) { return v; }
inline void warp_sync() {}
inline uint32_t warp_min(uint32_t v) { return v; }
#endif

enum : int { OK = 0, E_DST = 2, E_CORRUPT = 17, E_CHECKSUM = 18, E_UNSUPPORTED = 19 };

constexpr uint32_t MAGIC = 0xFD2FB528u;
constexpr uint32_t SKIP_MAGIC = 0x184D2A50u;  // low 4 bits: any
constexpr uint32_t BLOCK_MAX = 128 * 1024;
constexpr int LL_MAX_LOG = 9, OF_MAX_LOG = 8, ML_MAX_LOG = 9, HUF_MAX_LOG = 12;
constexpr int LL_MAX_SYM = 35, OF_MAX_SYM = 31, ML_MAX_SYM = 52;
constexpr int SEQ_BATCH = 64;
constexpr size_t LIT_SCRATCH = BLOCK_MAX + 64;  // bytes of literal scratch per warp

struct FseEntry {
    uint16_t base;  // next state base
    uint8_t sym;
    uint8_t nb;  // bits to read for the next state
};
// Huffman decoding table entry: symbol in bits 0-7, code length in 8-15.
typedef uint16_t HufEntry;

// Per-warp state that lives across the blocks of a frame (shared memory on
// the device).
struct Workspace {
    FseEntry ll[1 << LL_MAX_LOG];
    FseEntry ml[1 << ML_MAX_LOG];
    FseEntry of[1 << OF_MAX_LOG];
    HufEntry huf[1 << HUF_MAX_LOG];
    FseEntry wt[64];  // FSE table of the Huffman weights
    int16_t norm[256];
    uint16_t next[256];  // FSE table construction scratch
    uint8_t weights[256];
    uint32_t seq_ll[SEQ_BATCH], seq_ml[SEQ_BATCH], seq_of[SEQ_BATCH];
    uint64_t seq_pos[SEQ_BATCH];  // output position of each sequence's match
    uint32_t seq_lit[SEQ_BATCH];  // its literals' offset in the literal buffer
    uint8_t seq_state[SEQ_BATCH]; // match: 0 pending, 1 done, 2 ready for the whole warp
    uint32_t rep[3];
    int8_t ll_log, ml_log, of_log, huf_log;  // -1: no table yet
    uint16_t huf_nsym;  // symbols of the Huffman description
    int err;
    uint32_t nseq;      // sequences of the current batch
    uint32_t seq_done;  // the bitstream was consumed completely
};

// Huffman state of the block-parallel decoder (one per warp, shared memory):
// the members huf_read_table, huf_fill and huf_stream use, with a table of
// up to 2^TAB_LOG entries (decode_block fails a block whose table is larger).
template <int LOG>
struct HufWsT {
    static constexpr int TAB_LOG = LOG;
    HufEntry huf[1 << LOG];
    FseEntry wt[64];
    int16_t norm[256];
    uint16_t next[256];
    uint8_t weights[256];
    int8_t huf_log;
    uint16_t huf_nsym;
    int err;
};
typedef HufWsT<HUF_MAX_LOG> HufWs;  // any table

// ---- small helpers -------------------------------------------------------

ZHD uint32_t rd16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
ZHD uint32_t rd24(const uint8_t *p) { return rd16(p) | ((uint32_t)p[2] << 16); }
ZHD uint32_t rd32(const uint8_t *p) { return rd16(p) | (rd16(p + 2) << 16); }
ZHD uint64_t rd64(const uint8_t *p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

// 8 bytes to an 8-byte aligned address
ZHD void st_u64(uint8_t *p, uint64_t v) {
#if defined(__CUDA_ARCH__)
    *reinterpret_cast<uint64_t *>(p) = v;
#else
    for (int k = 0; k < 8; k++) p[k] = (uint8_t)(v >> (8 * k));
#endif
}

ZHD int highbit(uint32_t v) {  // index of the highest set bit, v > 0
#if defined(__CUDA_ARCH__)
    return 31 - __clz(v);
#else
    return 31 - __builtin_clz(v);
#endif
}

// 8 bytes at p (little endian); bytes at or past end read as zero.  On the
// device, two aligned 8-byte loads when both lie before end (an 8-byte
// aligned word never starts below an 8-byte aligned allocation).
ZHD uint64_t rd64_bounded(const uint8_t *p, const uint8_t *end) {
#if defined(__CUDA_ARCH__)
    const uintptr_t a = (uintptr_t)p & 7;
    const uint64_t *w = reinterpret_cast<const uint64_t *>(p - a);
    if ((const uint8_t *)(w + 2) <= end) {
        const uint64_t lo = w[0];
        return a ? (lo >> (8 * a)) | (w[1] << (64 - 8 * a)) : lo;
    }
#endif
    if (p + 8 <= end) return rd64(p);
    uint64_t v = 0;
    for (int i = 0; i < 8 && p + i < end; i++) v |= (uint64_t)p[i] << (8 * i);
    return v;
}

// Backward bit reader over [start, end): bits are taken from the top, bit
// pos - 1 first.  Reading below bit 0 yields zeros (pos goes negative),
// which callers treat as the reference's "overflow".
struct BitRev {
    const uint8_t *base, *end;
    int64_t pos;   // bits not yet consumed
    int64_t cbit;  // first bit held in cont
    uint64_t cont;

    ZHD bool init(const uint8_t *s, const uint8_t *e) {
        base = s;
        end = e;
        if (e <= s) return false;
        const uint8_t last = e[-1];
        if (last == 0) return false;  // no end mark
        pos = (int64_t)(e - s) * 8 - (8 - highbit(last));
        cbit = 1;  // forces a load
        cont = 0;
        reload();
        return true;
    }
    ZHD void reload() {
        int64_t b = pos >= 64 ? ((pos - 64 + 7) & ~(int64_t)7) : 0;
        cbit = b;
        cont = rd64_bounded(base + (b >> 3), end);
    }
    // n <= 56 bits
    ZHD uint64_t peek(int n) {
        if (n == 0) return 0;
        if (pos - n < cbit && cbit > 0) reload();  // after it, pos - n >= cbit or cbit == 0
        if (pos - n >= cbit) return (cont >> (pos - n - cbit)) & ((1ull << n) - 1);
        // below the first bit (cbit == 0): the bits left, shifted up, zeros below
        if (pos <= 0) return 0;
        return (cont & ((1ull << pos) - 1)) << (n - pos);
    }
    ZHD uint64_t read(int n) {
        const uint64_t v = peek(n);
        pos -= n;
        return v;
    }
    ZHD void skip(int n) { pos -= n; }
};

// Forward bit reader (FSE table descriptions): bit 0 of byte 0 first.
struct BitFwd {
    const uint8_t *base, *end;
    int64_t pos;
    ZHD uint64_t peek(int n) const {
        const int64_t byte = pos >> 3;
        const uint64_t v = rd64_bounded(base + byte, end) >> (pos & 7);
        return v & ((1ull << n) - 1);
    }
    ZHD void skip(int n) { pos += n; }
};

// ---- FSE -----------------------------------------------------------------

// FSE table description (RFC 8878 4.1.1; libzstd FSE_readNCount): the
// normalized counts of symbols 0..max_sym into norm, *log the accuracy log.
// Returns the bytes used, or -1 when the description is invalid.
ZCOLD int fse_read_ncount(const uint8_t *src, size_t len, int16_t *norm, int max_sym, int max_log,
                        int *log, int *nsym) {
    if (len < 1) return -1;
    BitFwd br{src, src + len, 0};
    const int al = (int)br.peek(4) + 5;
    br.skip(4);
    if (al > max_log) return -1;
    int remaining = (1 << al) + 1, threshold = 1 << al, nb = al + 1, sym = 0;
    bool prev0 = false;
    while (remaining > 1 && sym <= max_sym) {
        if (prev0) {
            int n0 = sym;
            for (;;) {
                const int r = (int)br.peek(2);
                br.skip(2);
                n0 += r;
                if (r != 3) break;
                if (br.pos > (int64_t)len * 8) return -1;
            }
            if (n0 > max_sym) return -1;
            while (sym < n0) norm[sym++] = 0;
            if (br.pos > (int64_t)len * 8) return -1;
            if (sym > max_sym) break;
        }
        const int mx = (2 * threshold - 1) - remaining;
        int count;
        const uint32_t bits = (uint32_t)br.peek(nb);
        if ((int)(bits & (threshold - 1)) < mx) {
            count = (int)(bits & (threshold - 1));
            br.skip(nb - 1);
        } else {
            count = (int)(bits & (2 * threshold - 1));
            if (count >= threshold) count -= mx;
            br.skip(nb);
        }
        count--;
        remaining -= count < 0 ? -count : count;
        norm[sym++] = (int16_t)count;
        prev0 = count == 0;
        while (remaining < threshold) {
            nb--;
            threshold >>= 1;
        }
        if (br.pos > (int64_t)len * 8) return -1;
    }
    if (remaining != 1 || sym > max_sym + 1) return -1;
    *log = al;
    *nsym = sym;
    const int64_t used = (br.pos + 7) >> 3;
    if (used > (int64_t)len) return -1;
    return (int)used;
}

// Decoding table from normalized counts (RFC 8878 4.1.1; libzstd
// FSE_buildDTable): low-probability symbols at the top, the others spread
// with step (size/2 + size/8 + 3), then each state's bits and base.
ZCOLD bool fse_build(FseEntry *t, const int16_t *norm, int nsym, int log, uint16_t *next) {
    const int size = 1 << log;
    int high = size - 1;
    for (int s = 0; s < nsym; s++) {
        if (norm[s] == -1) {
            t[high--].sym = (uint8_t)s;
            next[s] = 1;
        } else {
            next[s] = (uint16_t)norm[s];
        }
    }
    const int step = (size >> 1) + (size >> 3) + 3, mask = size - 1;
    int p = 0;
    for (int s = 0; s < nsym; s++) {
        for (int i = 0; i < norm[s]; i++) {
            t[p].sym = (uint8_t)s;
            do {
                p = (p + step) & mask;
            } while (p > high);
        }
    }
    if (p != 0) return false;
    for (int u = 0; u < size; u++) {
        const int s = t[u].sym;
        const uint32_t n = next[s]++;
        const int nb = log - highbit(n);
        t[u].nb = (uint8_t)nb;
        t[u].base = (uint16_t)((n << nb) - (uint32_t)size);
    }
    return true;
}

// One-symbol table (RLE mode)
ZHD void fse_rle(FseEntry *t, int sym) {
    t[0].sym = (uint8_t)sym;
    t[0].nb = 0;
    t[0].base = 0;
}

// Predefined distributions (RFC 8878 3.1.1.3.2.2).
// Constant tables: __constant__ memory on the device (a function-local
// array indexed at run time would be rebuilt on the stack at every call),
// plain constants on the host.
#if defined(__CUDACC__)
#define ZTAB(type, name, n, ...)                                \
    static __constant__ const type name##_dev[n] = __VA_ARGS__; \
    static constexpr type name##_host[n] = __VA_ARGS__;
#else
#define ZTAB(type, name, n, ...) static constexpr type name##_host[n] = __VA_ARGS__;
#endif
#if defined(__CUDA_ARCH__)
#define ZLOOK(name, i) name##_dev[i]
#else
#define ZLOOK(name, i) name##_host[i]
#endif

// Predefined distributions (RFC 8878 3.1.1.3.2.2).
ZTAB(int16_t, LL_DEFAULT, 36, {4, 3, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 2, 1, 1, 1, 2, 2,
                               2, 2, 2, 2, 2, 2, 2, 3, 2, 1, 1, 1, 1, 1, -1, -1, -1, -1})
ZTAB(int16_t, ML_DEFAULT, 53, {1, 4, 3, 2, 2, 2, 2, 2, 2, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                               1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                               1, 1, 1, 1, 1, 1, 1, 1, 1, 1, -1, -1, -1, -1, -1, -1, -1})
ZTAB(int16_t, OF_DEFAULT, 29, {1, 1, 1, 1, 1, 1, 2, 2, 2, 1, 1, 1, 1, 1, 1,
                               1, 1, 1, 1, 1, 1, 1, 1, 1, -1, -1, -1, -1, -1})
// Literal and match length codes (RFC 8878 3.1.1.3.2.1.1).
ZTAB(uint32_t, LL_BASE, 36, {0,  1,  2,  3,  4,   5,   6,   7,   8,    9,    10,   11,
                             12, 13, 14, 15, 16,  18,  20,  22,  24,   28,   32,   40,
                             48, 64, 128, 256, 512, 1024, 2048, 4096, 8192, 16384, 32768, 65536})
ZTAB(uint8_t, LL_BITS, 36, {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1,
                            1, 1, 2, 2, 3, 3, 4, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16})
ZTAB(uint32_t, ML_BASE, 53, {3,  4,  5,  6,  7,  8,  9,  10,  11,  12,  13,   14,   15,   16,
                             17, 18, 19, 20, 21, 22, 23, 24,  25,  26,  27,   28,   29,   30,
                             31, 32, 33, 34, 35, 37, 39, 41,  43,  47,  51,   59,   67,   83,
                             99, 131, 259, 515, 1027, 2051, 4099, 8195, 16387, 32771, 65539})
ZTAB(uint8_t, ML_BITS, 53, {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
                            0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1,
                            2, 2, 3, 3, 4, 4, 5, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16})

ZHD int16_t ll_default(int s) { return ZLOOK(LL_DEFAULT, s); }
ZHD int16_t ml_default(int s) { return ZLOOK(ML_DEFAULT, s); }
ZHD int16_t of_default(int s) { return ZLOOK(OF_DEFAULT, s); }
ZHD uint32_t ll_base(int c) { return ZLOOK(LL_BASE, c); }
ZHD int ll_bits(int c) { return ZLOOK(LL_BITS, c); }
ZHD uint32_t ml_base(int c) { return ZLOOK(ML_BASE, c); }
ZHD int ml_bits(int c) { return ZLOOK(ML_BITS, c); }

// ---- Huffman -------------------------------------------------------------

// Huffman tree description (RFC 8878 4.2.1; libzstd HUF_readStats +
// HUF_readDTableX1): weights (direct 4-bit, or FSE-compressed with two
// interleaved states), the implied last weight, then where each symbol's
// entries start in the single-symbol decoding table of 2^log entries
// (huf_fill writes the table).  Returns the bytes used, -1 if invalid.
// Lane 0 only.
template <class W>
ZCOLD int huf_read_table(W *ws, const uint8_t *src, size_t len) {
    if (len < 1) return -1;
    const int isz = src[0];
    int nw = 0;
    size_t used;
    if (isz >= 128) {
        nw = isz - 127;
        const size_t bytes = (size_t)(nw + 1) / 2;
        if (bytes + 1 > len) return -1;
        for (int n = 0; n < nw; n += 2) {
            const uint8_t b = src[1 + n / 2];
            ws->weights[n] = b >> 4;
            if (n + 1 < nw) ws->weights[n + 1] = b & 15;
        }
        used = bytes + 1;
    } else {
        if ((size_t)isz + 1 > len) return -1;
        int log = 0, nsym = 0;
        const int h = fse_read_ncount(src + 1, (size_t)isz, ws->norm, 255, 6, &log, &nsym);
        if (h < 0) return -1;
        if (!fse_build(ws->wt, ws->norm, nsym, log, ws->next)) return -1;
        BitRev br{};
        if (!br.init(src + 1 + h, src + 1 + isz)) return -1;
        uint32_t s1 = (uint32_t)br.read(log), s2 = (uint32_t)br.read(log);
        // libzstd FSE_decompress (two states): a symbol per state in turn
        // until a state update reads past the start of the stream, then the
        // other state's symbol ends the list.
        for (;;) {
            if (nw > 253) return -1;
            ws->weights[nw++] = ws->wt[s1].sym;
            s1 = ws->wt[s1].base + (uint32_t)br.read(ws->wt[s1].nb);
            if (br.pos < 0) {
                ws->weights[nw++] = ws->wt[s2].sym;
                break;
            }
            if (nw > 253) return -1;
            ws->weights[nw++] = ws->wt[s2].sym;
            s2 = ws->wt[s2].base + (uint32_t)br.read(ws->wt[s2].nb);
            if (br.pos < 0) {
                ws->weights[nw++] = ws->wt[s1].sym;
                break;
            }
        }
        used = (size_t)isz + 1;
    }
    // weight statistics and the implied last weight
    uint32_t rank[HUF_MAX_LOG + 2] = {0};
    uint32_t total = 0;
    for (int n = 0; n < nw; n++) {
        const int w = ws->weights[n];
        if (w > HUF_MAX_LOG) return -1;
        rank[w]++;
        total += (1u << w) >> 1;
    }
    if (total == 0) return -1;
    const int log = highbit(total) + 1;
    if (log > HUF_MAX_LOG) return -1;
    const uint32_t rest = (1u << log) - total;
    const int lastw = highbit(rest) + 1;
    if ((1u << highbit(rest)) != rest) return -1;
    if (nw > 255) return -1;
    ws->weights[nw] = (uint8_t)lastw;
    rank[lastw]++;
    if (rank[1] < 2 || (rank[1] & 1)) return -1;
    const int nsym = nw + 1;
    // single-symbol decoding table: symbols of weight w fill 2^(w-1) entries
    uint32_t start[HUF_MAX_LOG + 2];
    uint32_t next = 0;
    for (int w = 1; w <= log; w++) {
        start[w] = next;
        next += rank[w] << (w - 1);
    }
    // each symbol's first entry (the warp fills the table: huf_fill)
    for (int n = 0; n < nsym; n++) {
        const int w = ws->weights[n];
        ws->next[n] = (uint16_t)start[w];
        if (w) start[w] += (1u << w) >> 1;
    }
    ws->huf_nsym = (uint16_t)nsym;
    ws->huf_log = (int8_t)log;
    return (int)used;
}

// Decoding table of the description huf_read_table just read, filled by
// the warp: symbols of weight w take 2^(w-1) consecutive entries from their
// first entry on, each entry {symbol, code length log + 1 - w}.
template <class W>
ZHD void huf_fill(W *ws, int lane, int nl) {
    const int log = ws->huf_log, nsym = ws->huf_nsym;
    for (int n = 0; n < nsym; n++) {
        const int w = ws->weights[n];
        if (!w) continue;
        const uint32_t st = ws->next[n], cnt = (1u << w) >> 1;
        const HufEntry e = (HufEntry)(n | ((uint32_t)(log + 1 - w) << 8));
        for (uint32_t u = (uint32_t)lane; u < cnt; u += (uint32_t)nl) ws->huf[st + u] = e;
    }
}

// Backward reader over aligned 32-bit words (Huffman streams, sequence
// bitstreams).  Bits are numbered from base = s rounded down to 4 bytes; the
// stream holds bits [lo, top) and pos counts the bits not yet consumed.
// Words hi (index w, holding bit pos - 1) and lo_w (index w - 1) form a
// window of at least 33 unconsumed bits: a read of up to 31 bits, or two
// Huffman symbols of <= 12 bits, fit between window checks.  Bits below the
// stream read as zero (libzstd's reader zero-fills below its start) and pos
// then drops below lo; bits above pos are masked off.
struct BitWin {
    const uint8_t *s, *e;
    const uint32_t *base;
    int32_t lo, pos, w;
    uint32_t hi, lo_w, nx;  // words w, w - 1 and (loaded ahead) w - 2

    ZHD uint32_t word(int32_t i) const {
#if defined(__CUDA_ARCH__)
        // the aligned word holding a stream byte lies inside the allocation;
        // selects instead of branches (the lanes of a warp run 4 streams)
        uint32_t v = __ldg(base + (i < 0 ? 0 : i));
        v = i < 0 ? 0u : v;
#else
        if (i < 0) return 0;
        uint32_t v = 0;
        const uint8_t *wb = reinterpret_cast<const uint8_t *>(base) + 4 * (int64_t)i;
        for (int k = 0; k < 4; k++)
            if (wb + k >= s && wb + k < e) v |= (uint32_t)wb[k] << (8 * k);
#endif
        return v & (i == 0 ? ~0u << lo : ~0u);  // lo < 32: bits of the bytes before s
    }
    ZHD bool init(const uint8_t *start, const uint8_t *end) {
        if (end <= start) return false;
        const uint8_t last = end[-1];
        if (last == 0) return false;  // no end mark
        s = start;
        e = end;
        base = reinterpret_cast<const uint32_t *>((uintptr_t)start & ~(uintptr_t)3);
        lo = (int32_t)((uintptr_t)start & 3) * 8;
        pos = lo + (int32_t)(end - start) * 8 - (8 - highbit(last));
        w = (pos - 1) >> 5;
        hi = word(w);
        lo_w = word(w - 1);
        nx = word(w - 2);
        return true;
    }
    // the next n <= 31 bits (sh reaches 64 only for n == 0, masked to 0)
    ZHD uint32_t peek(int n) const {
        const uint32_t sh = (uint32_t)(pos - n - (w - 1) * 32) & 63;
        return (uint32_t)((((uint64_t)hi << 32) | lo_w) >> sh) & ((1u << n) - 1);
    }
    ZHD void slide() {
        // selects, not a branch: the lanes of a warp run different streams
        const bool c = pos <= w * 32;
        w -= c ? 1 : 0;
        hi = c ? lo_w : hi;
        lo_w = c ? nx : lo_w;
        nx = word(w - 2);
    }
    // the same while w >= 4: word w - 2 lies above the stream's first word
    // and needs no masking
    ZHD void slide_inner() {
        const bool c = pos <= w * 32;
        w -= c ? 1 : 0;
        hi = c ? lo_w : hi;
        lo_w = c ? nx : lo_w;
#if defined(__CUDA_ARCH__)
        nx = __ldg(base + (w - 2));
#else
        nx = word(w - 2);
#endif
    }
    // peek for 1 <= n <= 31 (the shift then stays below 64)
    ZHD uint32_t peek1(int n) const {
        const uint32_t sh = (uint32_t)(pos - n - (w - 1) * 32);
        return (uint32_t)((((uint64_t)hi << 32) | lo_w) >> sh) & ((1u << n) - 1);
    }
    ZHD uint32_t read(int n) {
        const uint32_t v = peek(n);
        pos -= n;
        slide();
        return v;
    }
};

// One Huffman stream of n symbols into out; false unless the stream is
// consumed exactly (libzstd HUF_decompress1X1: BIT_endOfDStream).
template <class W>
ZHD bool huf_stream(const W *ws, const uint8_t *s, const uint8_t *e, uint8_t *out,
                    uint32_t n) {
    BitWin br;
    if (!br.init(s, e)) return false;
    const int log = ws->huf_log;
    auto sym = [&]() -> uint32_t {
        const uint32_t d = ws->huf[br.peek(log)];
        br.pos -= (int32_t)(d >> 8);
        return d & 0xFF;
    };
    uint32_t i = 0;
    // single symbols up to an 8-byte aligned output address
    const uint32_t head = (uint32_t)((8 - ((uintptr_t)out & 7)) & 7);
    for (; i < n && i < head; i++) {
        out[i] = (uint8_t)sym();
        br.slide();
    }
    // 8 symbols per step while the window stays 4+ words above the stream's
    // start (8 symbols take at most 3 words)
    auto sym1 = [&]() -> uint32_t {
        const uint32_t d = ws->huf[br.peek1(log)];
        br.pos -= (int32_t)(d >> 8);
        return d & 0xFF;
    };
    for (; i + 8 <= n && br.w >= 8; i += 8) {
        uint32_t v0 = 0, v1 = 0;
ZUNROLL
        for (int k = 0; k < 4; k += 2) {
            const uint32_t a = sym1();
            const uint32_t b = sym1();
            br.slide_inner();
            v0 |= (a | (b << 8)) << (8 * k);
        }
ZUNROLL
        for (int k = 0; k < 4; k += 2) {
            const uint32_t a = sym1();
            const uint32_t b = sym1();
            br.slide_inner();
            v1 |= (a | (b << 8)) << (8 * k);
        }
        st_u64(out + i, (uint64_t)v0 | ((uint64_t)v1 << 32));
    }
    for (; i < n; i++) {
        out[i] = (uint8_t)sym();
        br.slide();
    }
    return br.pos == br.lo;
}

// ---- XXH64 (content checksum) --------------------------------------------

constexpr uint64_t P64_1 = 11400714785074694791ull, P64_2 = 14029467366897019727ull,
                   P64_3 = 1609587929392839161ull, P64_4 = 9650029242287828579ull,
                   P64_5 = 2870177450012600261ull;
ZHD uint64_t rotl64(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }
ZHD uint64_t xxh_round(uint64_t acc, uint64_t in) {
    acc += in * P64_2;
    return rotl64(acc, 31) * P64_1;
}
ZHD uint64_t xxh_merge(uint64_t acc, uint64_t v) {
    acc ^= xxh_round(0, v);
    return acc * P64_1 + P64_4;
}

// XXH64 with seed 0 of [p, p + n); the stripe accumulators run on lanes
// 0..3 (nl >= 4) or all on lane 0.  Result valid on lane 0; acc is a
// 4-entry scratch shared by the warp.
ZHD uint64_t xxh64(const uint8_t *p, uint64_t n, int lane, int nl, uint64_t *acc, uint64_t *stage) {
    const uint64_t stripes = n / 32;
    const uint8_t *pe = p + n;
    auto init = [](int a) -> uint64_t {
        return a == 0 ? P64_1 + P64_2 : (a == 1 ? P64_2 : (a == 2 ? 0 : 0 - P64_1));
    };
#if defined(__CUDA_ARCH__)
    if (n >= 32 && nl == 32) {
        // 1 KiB chunks (32 stripes) staged in shared memory: every lane
        // loads 32 bytes of chunk c + 1 while lanes 0-3 run chunk c, so the
        // rounds never wait on a global load
        const uint64_t nch = stripes / 32;
        uint64_t v = init(lane & 3), r[4];
        ZUNROLL
        for (int k = 0; k < 4; k++) r[k] = nch ? rd64_bounded(p + 32 * lane + 8 * k, pe) : 0;
        for (uint64_t c = 0; c < nch; c++) {
            warp_sync();
            ZUNROLL
            for (int k = 0; k < 4; k++) stage[4 * lane + k] = r[k];
            warp_sync();
            if (c + 1 < nch) {
                const uint8_t *q = p + 1024 * (c + 1) + 32 * lane;
                ZUNROLL
                for (int k = 0; k < 4; k++) r[k] = rd64_bounded(q + 8 * k, pe);
            }
            if (lane < 4)
                for (int t = 0; t < 32; t++) v = xxh_round(v, stage[4 * t + lane]);
        }
        if (lane < 4) {
            for (uint64_t t = 32 * nch; t < stripes; t++) v = xxh_round(v, rd64_bounded(p + 32 * t + 8 * lane, pe));
            acc[lane] = v;
        }
    } else
#endif
    if (n >= 32) {
        for (int a = lane; a < 4; a += nl) {
            uint64_t v = init(a);
            for (uint64_t s = 0; s < stripes; s++) v = xxh_round(v, rd64_bounded(p + 32 * s + 8 * a, pe));
            acc[a] = v;
        }
    }
    warp_sync();
    uint64_t h = 0;
    if (lane == 0) {
        if (n >= 32) {
            h = rotl64(acc[0], 1) + rotl64(acc[1], 7) + rotl64(acc[2], 12) + rotl64(acc[3], 18);
            for (int a = 0; a < 4; a++) h = xxh_merge(h, acc[a]);
        } else {
            h = P64_5;
        }
        h += n;
        const uint8_t *q = p + 32 * stripes;
        uint64_t r = n - 32 * stripes;
        while (r >= 8) {
            h ^= xxh_round(0, rd64(q));
            h = rotl64(h, 27) * P64_1 + P64_4;
            q += 8;
            r -= 8;
        }
        if (r >= 4) {
            h ^= (uint64_t)rd32(q) * P64_1;
            h = rotl64(h, 23) * P64_2 + P64_3;
            q += 4;
            r -= 4;
        }
        while (r) {
            h ^= (uint64_t)(*q) * P64_5;
            h = rotl64(h, 11) * P64_1;
            q++;
            r--;
        }
        h ^= h >> 33;
        h *= P64_2;
        h ^= h >> 29;
        h *= P64_3;
        h ^= h >> 32;
    }
    return h;
}

// ---- sequences -----------------------------------------------------------

// Table of one sequence field for its compression mode (RFC 8878
// 3.1.1.3.2.1): 0 predefined, 1 RLE (one symbol byte), 2 FSE-compressed
// (a table description), 3 repeat the previous table.  Returns bytes used
// or -1.  Lane 0 only.
ZCOLD int seq_table(Workspace *ws, int field, int mode, const uint8_t *src, size_t len) {
    FseEntry *t = field == 0 ? ws->ll : (field == 1 ? ws->of : ws->ml);
    int8_t *lg = field == 0 ? &ws->ll_log : (field == 1 ? &ws->of_log : &ws->ml_log);
    const int max_sym = field == 0 ? LL_MAX_SYM : (field == 1 ? OF_MAX_SYM : ML_MAX_SYM);
    const int max_log = field == 0 ? LL_MAX_LOG : (field == 1 ? OF_MAX_LOG : ML_MAX_LOG);
    if (mode == 0) {
        const int n = field == 0 ? 36 : (field == 1 ? 29 : 53);
        for (int s = 0; s < n; s++)
            ws->norm[s] = field == 0 ? ll_default(s) : (field == 1 ? of_default(s) : ml_default(s));
        const int log = field == 1 ? 5 : 6;
        if (!fse_build(t, ws->norm, n, log, ws->next)) return -1;
        *lg = (int8_t)log;
        return 0;
    }
    if (mode == 1) {
        if (len < 1 || src[0] > max_sym) return -1;
        fse_rle(t, src[0]);
        *lg = 0;
        return 1;
    }
    if (mode == 2) {
        int log = 0, nsym = 0;
        const int h = fse_read_ncount(src, len, ws->norm, max_sym, max_log, &log, &nsym);
        if (h < 0) return -1;
        if (!fse_build(t, ws->norm, nsym, log, ws->next)) return -1;
        *lg = (int8_t)log;
        return h;
    }
    return *lg < 0 ? -1 : 0;  // repeat: needs an earlier table
}

// ---- the decoder ---------------------------------------------------------

struct Job {
    const uint8_t *src;
    uint64_t len;
    uint8_t *dst;
    uint64_t cap;
    uint8_t *lit;  // LIT_SCRATCH bytes of the warp
};

struct Result {
    int code;
    uint64_t pos;      // input offset of the failing frame or block
    uint64_t written;  // output bytes
};

// Cooperative copies (lanes lane, lane + nl, ...): n bytes from s to d (no
// overlap).
ZHD void coop_copy(uint8_t *d, const uint8_t *s, uint64_t n, int lane, int nl) {
#if defined(__CUDA_ARCH__)
    // bytes up to a 16-byte aligned destination, then 16-byte stores of
    // source words realigned by funnel shifts (4 chunks in flight per lane),
    // then the tail.  A source word read is an aligned word holding at least
    // one byte of [s, s + n).
    const uint64_t head = ((16 - ((uintptr_t)d & 15)) & 15) < n ? ((16 - ((uintptr_t)d & 15)) & 15) : n;
    for (uint64_t i = (uint64_t)lane; i < head; i += (uint64_t)nl) d[i] = s[i];
    const uint64_t nch = (n - head) / 16;
    if (nch) {
        const uint8_t *s1 = s + head;
        uint4 *d1 = reinterpret_cast<uint4 *>(d + head);
        const uint32_t sh = (uint32_t)((uintptr_t)s1 & 3) * 8;
        const uint32_t *w = reinterpret_cast<const uint32_t *>(s1 - ((uintptr_t)s1 & 3));
        auto chunk = [&](uint64_t c, uint32_t *v) {
            const uint32_t *q = w + 4 * c;
            const uint32_t a = q[0], b = q[1], e = q[2], f = q[3], g = sh ? q[4] : 0u;
            v[0] = __funnelshift_r(a, b, sh);
            v[1] = __funnelshift_r(b, e, sh);
            v[2] = __funnelshift_r(e, f, sh);
            v[3] = __funnelshift_r(f, g, sh);
        };
        const uint64_t step = (uint64_t)nl * 4;
        uint64_t c = (uint64_t)lane;
        for (; c + 3 * (uint64_t)nl < nch; c += step) {
            uint32_t v[4][4];
ZUNROLL
            for (int k = 0; k < 4; k++) chunk(c + (uint64_t)k * nl, v[k]);
ZUNROLL
            for (int k = 0; k < 4; k++) d1[c + (uint64_t)k * nl] = make_uint4(v[k][0], v[k][1], v[k][2], v[k][3]);
        }
        for (; c < nch; c += (uint64_t)nl) {
            uint32_t v[4];
            chunk(c, v);
            d1[c] = make_uint4(v[0], v[1], v[2], v[3]);
        }
    }
    for (uint64_t i = head + 16 * nch + (uint64_t)lane; i < n; i += (uint64_t)nl) d[i] = s[i];
#else
    for (uint64_t i = (uint64_t)lane; i < n; i += (uint64_t)nl) d[i] = s[i];
#endif
}

ZHD void coop_fill(uint8_t *d, uint8_t v, uint64_t n, int lane, int nl) {
    for (uint64_t i = (uint64_t)lane; i < n; i += (uint64_t)nl) d[i] = v;
}

// Match: ml bytes at d from d - off (off >= 1); with off < ml the bytes
// repeat the period-off pattern, read from before d, each lane 16
// consecutive bytes per step with all loads before the stores.
constexpr int CCH = 16;
ZHD void coop_match(uint8_t *d, uint64_t off, uint64_t ml, int lane, int nl) {
    const uint8_t *s = d - off;
    if (off >= ml) {
        coop_copy(d, s, ml, lane, nl);
        return;
    }
    for (uint64_t i = (uint64_t)lane * CCH; i < ml; i += (uint64_t)nl * CCH) {
        uint8_t t[CCH];
        const uint64_t m = ml - i < (uint64_t)CCH ? ml - i : (uint64_t)CCH;
        uint64_t j = i % off;
ZUNROLL
        for (int k = 0; k < CCH; k++) {
            if ((uint64_t)k < m) t[k] = s[j];
            if (++j == off) j = 0;
        }
ZUNROLL
        for (int k = 0; k < CCH; k++)
            if ((uint64_t)k < m) d[i + k] = t[k];
    }
}

// The Huffman-coded literals (RFC 8878 3.1.1.3.1.6) of [p, pe): one stream,
// or a 6-byte jump table and four streams of (regen + 3) / 4 symbols (the
// last one the rest), into out.  False unless every stream decodes exactly.
// All lanes call it; lanes 0-3 decode a stream each.
template <class W>
ZHD bool lit_streams(W *ws, const uint8_t *p, const uint8_t *pe, int nstreams, uint32_t regen,
                     uint8_t *out, int lane, int nl) {
    if (nstreams == 1) {
        if (lane == 0) ws->err = huf_stream(ws, p, pe, out, regen) ? OK : E_CORRUPT;
    } else {
        if (pe - p < 6) return false;
        const uint32_t s1 = rd16(p), s2 = rd16(p + 2), s3 = rd16(p + 4);
        const uint8_t *q = p + 6;
        const uint64_t total = (uint64_t)(pe - q);
        if ((uint64_t)s1 + s2 + s3 > total) return false;
        const uint32_t seg = (regen + 3) / 4;
        if (regen < 6 || 3 * seg > regen) return false;  // libzstd: >= 6 for 4 streams
        const uint8_t *st[5] = {q, q + s1, q + s1 + s2, q + s1 + s2 + s3, pe};
        if (lane == 0) ws->err = OK;
        warp_sync();
        for (int k = lane; k < 4; k += nl) {
            const uint32_t n = k < 3 ? seg : regen - 3 * seg;
            if (!huf_stream(ws, st[k], st[k + 1], out + (uint64_t)k * seg, n)) ws->err = E_CORRUPT;
        }
    }
    warp_sync();
    const bool ok = ws->err == OK;
    warp_sync();
    return ok;
}

// Literals section header (RFC 8878 3.1.1.3.1.1) of a compressed block of
// bsize bytes at b.  False when it is invalid or does not fit the block.
struct LitHdr {
    int ltype;         // 0 raw, 1 RLE, 2 compressed, 3 treeless
    int nstreams;      // Huffman streams (1 or 4)
    uint32_t regen;    // literal bytes
    uint32_t csize;    // compressed bytes (types 2, 3)
    uint32_t hs;       // header bytes
    uint32_t lsec;     // bytes of the whole literals section
};
ZHD bool lit_header(const uint8_t *b, uint32_t bsize, LitHdr *h) {
    if (bsize < 1) return false;
    const int ltype = b[0] & 3, sfmt = (b[0] >> 2) & 3;
    uint32_t regen = 0, csize = 0, hs = 0;
    int nstreams = 1;
    if (ltype < 2) {  // raw / RLE
        if (sfmt == 0 || sfmt == 2) {
            hs = 1;
            regen = b[0] >> 3;
        } else if (sfmt == 1) {
            hs = 2;
            if (bsize < 2) return false;
            regen = (b[0] >> 4) | ((uint32_t)b[1] << 4);
        } else {
            hs = 3;
            if (bsize < 3) return false;
            regen = (b[0] >> 4) | ((uint32_t)b[1] << 4) | ((uint32_t)b[2] << 12);
        }
    } else {  // compressed / treeless
        if (sfmt < 2) {
            hs = 3;
            if (bsize < 3) return false;
            const uint32_t v = rd24(b);
            regen = (v >> 4) & 0x3FF;
            csize = (v >> 14) & 0x3FF;
            nstreams = sfmt == 0 ? 1 : 4;
        } else if (sfmt == 2) {
            hs = 4;
            if (bsize < 4) return false;
            const uint32_t v = rd32(b);
            regen = (v >> 4) & 0x3FFF;
            csize = (v >> 18) & 0x3FFF;
            nstreams = 4;
        } else {
            hs = 5;
            if (bsize < 5) return false;
            const uint64_t v = (uint64_t)rd32(b) | ((uint64_t)b[4] << 32);
            regen = (uint32_t)((v >> 4) & 0x3FFFF);
            csize = (uint32_t)((v >> 22) & 0x3FFFF);
            nstreams = 4;
        }
    }
    if (regen > BLOCK_MAX) return false;
    const uint32_t lsec = ltype == 0 ? hs + regen : (ltype == 1 ? hs + 1 : hs + csize);
    if (lsec > bsize || (ltype >= 2 && csize == 0)) return false;
    *h = LitHdr{ltype, nstreams, regen, csize, hs, lsec};
    return true;
}

// A compressed block (RFC 8878 3.1.1.3) of bsize bytes at b, its output
// appended at out (frame output starts at fstart).  Returns an error code.
// prelit: the block's Huffman literals, already decoded (the Huffman table
// is then left as it was).
ZHD int decode_compressed_block(Workspace *ws, const Job &job, const uint8_t *b, uint32_t bsize,
                                uint64_t fstart, uint64_t *out, int lane, int nl,
                                const uint8_t *prelit = nullptr) {
    // ---- literals section header
    LitHdr h;
    if (!lit_header(b, bsize, &h)) return E_CORRUPT;
    const int ltype = h.ltype, nstreams = h.nstreams;
    const uint32_t regen = h.regen, csize = h.csize, hs = h.hs;
    const uint8_t *lit = nullptr;  // the literals, or null for RLE
    uint8_t rle_byte = 0;
    const uint32_t lsec = h.lsec;  // bytes of the literals section
    if (ltype == 0) {
        lit = b + hs;
    } else if (ltype == 1) {
        rle_byte = b[hs];
    } else if (prelit) {  // Huffman literals decoded beforehand
        lit = prelit;
    } else {
        const uint8_t *p = b + hs, *pe = b + hs + csize;
        if (lane == 0) {
            ws->err = OK;
            if (ltype == 2) {
                const int used = huf_read_table(ws, p, (size_t)(pe - p));
                if (used < 0) ws->err = E_CORRUPT;
                else p += used;
            } else if (ws->huf_log < 0) {
                ws->err = E_CORRUPT;  // treeless without an earlier table
            }
            ws->seq_ll[0] = (uint32_t)(p - b);  // where the streams start
        }
        warp_sync();
        if (ws->err) return ws->err;
        p = b + ws->seq_ll[0];
        warp_sync();
        if (ltype == 2) {
            huf_fill(ws, lane, nl);
            warp_sync();
        }
        // a block whose sequence section is a lone zero byte (no sequences)
        // is its literals: they are decoded straight into the output
        const bool direct = lsec + 1 == bsize && b[lsec] == 0 && *out + regen <= job.cap;
        uint8_t *ld = direct ? job.dst + *out : job.lit;
        if (!lit_streams(ws, p, pe, nstreams, regen, ld, lane, nl)) return E_CORRUPT;
        if (direct) {
            *out += regen;
            return OK;
        }
        lit = job.lit;
    }
    // ---- sequences section (3.1.1.3.2)
    const uint8_t *s = b + lsec, *se = b + bsize;
    if (s >= se) return E_CORRUPT;
    uint32_t nseq;
    if (s[0] < 128) {
        nseq = s[0];
        s += 1;
    } else if (s[0] < 255) {
        if (se - s < 2) return E_CORRUPT;
        nseq = ((uint32_t)(s[0] - 128) << 8) | s[1];
        s += 2;
    } else {
        if (se - s < 3) return E_CORRUPT;
        nseq = (uint32_t)s[1] + ((uint32_t)s[2] << 8) + 0x7F00;
        s += 3;
    }
    uint64_t o = *out;
    uint32_t lused = 0;
    if (nseq == 0) {
        if (s != se) return E_CORRUPT;
    } else {
        if (s >= se) return E_CORRUPT;
        const int modes = s[0];
        if (modes & 3) return E_CORRUPT;
        s++;
        if (lane == 0) {
            ws->err = OK;
            const int m[3] = {modes >> 6, (modes >> 4) & 3, (modes >> 2) & 3};  // LL, OF, ML
            for (int f = 0; f < 3 && !ws->err; f++) {
                const int h = seq_table(ws, f, m[f], s, (size_t)(se - s));
                if (h < 0) ws->err = E_CORRUPT;
                else s += h;
            }
            ws->seq_ll[0] = (uint32_t)(s - b);
        }
        warp_sync();
        if (ws->err) return ws->err;
        s = b + ws->seq_ll[0];
        warp_sync();
        // lane 0 decodes batches of sequences; the warp executes them
        BitWin br{};
        uint32_t sll = 0, sof = 0, sml = 0;
        if (lane == 0) {
            ws->err = br.init(s, se) ? OK : E_CORRUPT;
            if (!ws->err) {
                sll = (uint32_t)br.read(ws->ll_log);
                sof = (uint32_t)br.read(ws->of_log);
                sml = (uint32_t)br.read(ws->ml_log);
            }
        }
        warp_sync();
        if (ws->err) return ws->err;
        for (uint32_t done = 0; done < nseq;) {
            const uint32_t nb = nseq - done < (uint32_t)SEQ_BATCH ? nseq - done : (uint32_t)SEQ_BATCH;
            // lane 0 decodes the batch and places each sequence, checking
            // in sequence order (the first failing sequence decides the error)
            if (lane == 0) {
                uint32_t r0 = ws->rep[0], r1 = ws->rep[1], r2 = ws->rep[2];
                for (uint32_t i = 0; i < nb; i++) {
                    const FseEntry eo = ws->of[sof], em = ws->ml[sml], el = ws->ll[sll];
                    const int oc = eo.sym, mc = em.sym, lc = el.sym;
                    if (oc > OF_MAX_SYM) { ws->err = E_CORRUPT; break; }
                    const uint64_t ofv = (1ull << oc) + br.read(oc);
                    // the match- then literal-length extra bits, in one read
                    // when they fit (a read takes at most 31 bits)
                    const int mb = ml_bits(mc), lb = ll_bits(lc);
                    uint32_t mx, lx;
                    if (mb + lb <= 31) {
                        const uint32_t x = br.read(mb + lb);
                        mx = x >> lb;
                        lx = x & ((1u << lb) - 1);
                    } else {
                        mx = br.read(mb);
                        lx = br.read(lb);
                    }
                    const uint32_t ml = ml_base(mc) + mx;
                    const uint32_t ll = ll_base(lc) + lx;
                    uint64_t off;
                    if (ofv > 3) {
                        off = ofv - 3;
                        r2 = r1;
                        r1 = r0;
                        r0 = (uint32_t)off;
                    } else {
                        const uint32_t idx = (uint32_t)ofv - 1 + (ll == 0 ? 1u : 0u);
                        if (idx == 0) {
                            off = r0;
                        } else {
                            uint64_t t = idx == 3 ? (uint64_t)r0 - 1 : (idx == 1 ? r1 : r2);
                            if (t == 0) t = ~0ull;  // invalid, caught below
                            if (idx != 1) r2 = r1;
                            r1 = r0;
                            r0 = (uint32_t)t;
                            off = t;
                        }
                    }
                    const uint32_t of32 = off > 0xFFFFFFFFull ? 0xFFFFFFFFu : (uint32_t)off;
                    if ((uint64_t)lused + ll > regen) { ws->err = E_CORRUPT; break; }
                    if (o + ll + ml > job.cap) { ws->err = E_DST; break; }
                    ws->seq_ll[i] = ll;
                    ws->seq_ml[i] = ml;
                    ws->seq_of[i] = of32;
                    ws->seq_lit[i] = lused;
                    ws->seq_pos[i] = o + ll;
                    ws->seq_state[i] = 0;
                    o += ll;
                    lused += ll;
                    if (of32 == 0 || (uint64_t)of32 > o - fstart) { ws->err = E_CORRUPT; break; }
                    o += ml;
                    if (done + i + 1 < nseq) {  // state updates LL, ML, OF: one read of <= 26 bits
                        const uint32_t x = br.read(el.nb + em.nb + eo.nb);
                        sll = el.base + (x >> (em.nb + eo.nb));
                        sml = em.base + ((x >> eo.nb) & ((1u << em.nb) - 1));
                        sof = eo.base + (x & ((1u << eo.nb) - 1));
                    }
                }
                ws->rep[0] = r0;
                ws->rep[1] = r1;
                ws->rep[2] = r2;
                if (!ws->err && done + nb == nseq && br.pos > br.lo) ws->err = E_CORRUPT;
            }
            o = bcast0(o);
            lused = (uint32_t)bcast0(lused);
            warp_sync();
            if (ws->err) return ws->err;
            warp_sync();
            // literals: a lane per sequence (they never overlap)
            for (uint32_t i = (uint32_t)lane; i < nb; i += (uint32_t)nl) {
                const uint32_t ll = ws->seq_ll[i];
                uint8_t *d = job.dst + ws->seq_pos[i] - ll;
                if (lit) coop_copy(d, lit + ws->seq_lit[i], ll, 0, 1);
                else coop_fill(d, rle_byte, ll, 0, 1);
            }
            warp_sync();
            // matches in waves: a match whose source bytes all lie below the
            // first pending match's output is final-sourced and runs now (on
            // its lane, or on the whole warp when long); the first pending
            // match itself always qualifies
            for (;;) {
                uint32_t mine = 0xFFFFFFFFu;
                for (uint32_t i = (uint32_t)lane; i < nb; i += (uint32_t)nl)
                    if (ws->seq_state[i] == 0 && i < mine) mine = i;
                const uint32_t fp = warp_min(mine);
                if (fp == 0xFFFFFFFFu) break;
                const uint64_t limit = ws->seq_pos[fp];
                for (uint32_t i = (uint32_t)lane; i < nb; i += (uint32_t)nl) {
                    if (ws->seq_state[i] != 0) continue;
                    const uint64_t mp = ws->seq_pos[i], off = ws->seq_of[i], ml = ws->seq_ml[i];
                    const uint64_t hi = off >= ml ? mp - off + ml : mp;  // source bytes needed
                    if (hi > limit) continue;
                    if (ml > 64) {
                        ws->seq_state[i] = 2;
                    } else {
                        coop_match(job.dst + mp, off, ml, 0, 1);
                        ws->seq_state[i] = 1;
                    }
                }
                warp_sync();
                for (uint32_t i = fp; i < nb; i++) {
                    if (ws->seq_state[i] != 2) continue;
                    coop_match(job.dst + ws->seq_pos[i], ws->seq_of[i], ws->seq_ml[i], lane, nl);
                    warp_sync();
                    if (lane == 0) ws->seq_state[i] = 1;
                }
                warp_sync();
            }
            done += nb;
            warp_sync();
        }
    }
    // the rest of the literals
    const uint32_t rest = regen - lused;
    if (o + rest > job.cap) return E_DST;
    if (lit) coop_copy(job.dst + o, lit + lused, rest, lane, nl);
    else coop_fill(job.dst + o, rle_byte, rest, lane, nl);
    o += rest;
    if (o - *out > BLOCK_MAX) return E_CORRUPT;
    *out = o;
    warp_sync();
    return OK;
}

// Every frame of [src, src + len) (RFC 8878 3.1): skippable frames skipped,
// zstd frames decoded in turn into dst.  ws must be private to the warp.
ZHD Result decode(Workspace *ws, const Job &job, int lane, int nl, uint64_t *acc) {
    Result r{OK, 0, 0};
    const uint8_t *src = job.src;
    uint64_t ip = 0, o = 0;
    // an empty input decodes to nothing (libzstd ZSTD_decompress)
    while (ip < job.len) {
        r.pos = ip;
        if (job.len - ip < 4) { r.code = E_CORRUPT; return r; }
        const uint32_t magic = rd32(src + ip);
        if ((magic & 0xFFFFFFF0u) == SKIP_MAGIC) {
            if (job.len - ip < 8) { r.code = E_CORRUPT; return r; }
            const uint64_t sz = rd32(src + ip + 4);
            if (job.len - ip - 8 < sz) { r.code = E_CORRUPT; return r; }
            ip += 8 + sz;
            continue;
        }
        if (magic != MAGIC) { r.code = E_CORRUPT; return r; }
        // ---- frame header (3.1.1.1)
        uint64_t p = ip + 4;
        if (p >= job.len) { r.code = E_CORRUPT; return r; }
        const int fhd = src[p++];
        const int fcs_flag = fhd >> 6, single = (fhd >> 5) & 1, cksum = (fhd >> 2) & 1;
        const int dict_flag = fhd & 3;
        if (fhd & 0x08) { r.code = E_CORRUPT; return r; }  // reserved bit
        const int dict_bytes = dict_flag == 0 ? 0 : (dict_flag == 1 ? 1 : (dict_flag == 2 ? 2 : 4));
        const int fcs_bytes = fcs_flag == 0 ? (single ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
        const uint64_t hlen = (uint64_t)(single ? 0 : 1) + dict_bytes + fcs_bytes;
        if (job.len - p < hlen) { r.code = E_CORRUPT; return r; }
        if (!single) {  // window descriptor: only its exponent is checked
            const int wlog = 10 + (src[p++] >> 3);
            if (wlog > 31) { r.code = E_UNSUPPORTED; return r; }
        }
        uint64_t dict = 0;
        for (int i = 0; i < dict_bytes; i++) dict |= (uint64_t)src[p + i] << (8 * i);
        p += dict_bytes;
        if (dict) { r.code = E_UNSUPPORTED; return r; }  // no dictionaries here
        uint64_t fcs = 0;
        bool has_fcs = fcs_bytes > 0;
        for (int i = 0; i < fcs_bytes; i++) fcs |= (uint64_t)src[p + i] << (8 * i);
        if (fcs_bytes == 2) fcs += 256;
        p += fcs_bytes;
        // fresh per frame: repeat offsets and tables
        if (lane == 0) {
            ws->rep[0] = 1;
            ws->rep[1] = 4;
            ws->rep[2] = 8;
            ws->ll_log = ws->ml_log = ws->of_log = ws->huf_log = -1;
        }
        warp_sync();
        const uint64_t fstart = o;
        // ---- blocks (3.1.1.2)
        for (;;) {
            r.pos = p;
            if (job.len - p < 3) { r.code = E_CORRUPT; return r; }
            const uint32_t bh = rd24(src + p);
            p += 3;
            const int last = bh & 1, type = (bh >> 1) & 3;
            const uint32_t bsize = bh >> 3;
            // libzstd: a compressed block is smaller than 128 KiB
            if (type == 3 || bsize > BLOCK_MAX || (type == 2 && bsize == BLOCK_MAX)) {
                r.code = E_CORRUPT;
                return r;
            }
            if (type == 0) {
                if (job.len - p < bsize) { r.code = E_CORRUPT; return r; }
                if (o + bsize > job.cap) { r.code = E_DST; return r; }
                coop_copy(job.dst + o, src + p, bsize, lane, nl);
                o += bsize;
                p += bsize;
            } else if (type == 1) {
                if (job.len - p < 1) { r.code = E_CORRUPT; return r; }
                if (o + bsize > job.cap) { r.code = E_DST; return r; }
                coop_fill(job.dst + o, src[p], bsize, lane, nl);
                o += bsize;
                p += 1;
            } else {
                if (job.len - p < bsize) { r.code = E_CORRUPT; return r; }
                const int e = decode_compressed_block(ws, job, src + p, bsize, fstart, &o, lane, nl);
                if (e) { r.code = e; r.written = o; return r; }
                p += bsize;
            }
            warp_sync();
            if (last) break;
        }
        if (has_fcs && o - fstart != fcs) { r.code = E_CORRUPT; r.pos = ip; return r; }
        if (cksum) {
            if (job.len - p < 4) { r.code = E_CORRUPT; return r; }
            // the frame's tables are dead at its end: their space stages the hash input
            const uint64_t h = xxh64(job.dst + fstart, o - fstart, lane, nl, acc,
                                     reinterpret_cast<uint64_t *>(ws->huf));
            if (lane == 0) ws->err = (uint32_t)h == rd32(src + p) ? OK : E_CHECKSUM;
            warp_sync();
            if (ws->err) { r.code = ws->err; r.pos = p; return r; }
            p += 4;
        }
        ip = p;
    }
    r.written = o;
    return r;
}

// ---- block-parallel frames -----------------------------------------------
//
// Every block of a frame written by zstd's encoder regenerates one block
// size, min(128 KiB, window), except the last, which regenerates the rest of
// the frame content size: so its blocks decode independently.  The plan
// below walks the block headers (one thread per job) and lists each block
// with its output offset and the Huffman description it uses (its own, or
// for treeless literals the last one before it).  Raw, RLE and
// sequence-free compressed blocks (whose sizes the headers give) go to the
// block kernel; blocks with sequences (taken to regenerate one block size)
// are decoded after them, in order, by the frame kernel, which carries the
// repeat offsets and sequence tables from one to the next and checks each
// size.  A job that is not one frame of that form, a block that fails, or a
// size that differs sends the job through decode() whole, which also gives
// every error its serial code and position.

struct BlockDesc {
    uint64_t src;   // block content offset in the job's input
    uint64_t out;   // output offset in the job's output
    uint64_t tbl;   // Huffman description offset in the job's input (types 2, 3)
    uint32_t job;
    uint32_t meta;  // bits 0-17 content bytes (RLE: output bytes), 18-19 block
                    // type (3: no block), 20-27 description bytes, 28: has
                    // sequences
    uint32_t slot;  // blocks with sequences: literal slot the block kernel
                    // decodes the Huffman literals into, or ~0
    uint32_t pad;
};
constexpr uint32_t META_SEQ = 1u << 28;

struct JobPlan {
    uint64_t total;    // output bytes
    uint64_t ckpos;    // input offset of the content checksum, or ~0
    uint64_t lastpos;  // input offset of the last block header
    uint32_t mode;     // 1: block-parallel
    uint32_t fail;     // set when a block did not decode
    uint32_t base;     // its first block descriptor
    uint32_t count;    // its blocks
    uint32_t nseq;     // of them with sequences
    uint32_t bsz;      // one block size (the regenerated size of a block with sequences)
};

// Bytes of the Huffman description starting with byte hb (RFC 8878 4.2.1).
ZHD uint32_t huf_desc_bytes(uint8_t hb) {
    return hb < 128 ? 1u + hb : 1u + ((uint32_t)(hb - 127) + 1) / 2;
}

// Walks the single zstd frame of a job.  True when it is block-parallel;
// *count = its blocks, written to d when d is not null.
ZHD bool plan_job(const uint8_t *src, uint64_t len, uint64_t cap, uint32_t job, JobPlan *jp,
                  BlockDesc *d, uint32_t *count) {
    *count = 0;
    if (len < 4 || rd32(src) != MAGIC) return false;
    uint64_t p = 4;
    if (p >= len) return false;
    const int fhd = src[p++];
    const int fcs_flag = fhd >> 6, single = (fhd >> 5) & 1, cksum = (fhd >> 2) & 1;
    if ((fhd & 0x08) || (fhd & 3)) return false;  // reserved bit, dictionary id
    const int fcs_bytes = fcs_flag == 0 ? (single ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
    if (len - p < (uint64_t)(single ? 0 : 1) + fcs_bytes) return false;
    uint64_t window = 0;
    if (!single) {
        const int wd = src[p++], wlog = 10 + (wd >> 3);
        if (wlog > 31) return false;
        window = (1ull << wlog) + ((1ull << wlog) >> 3) * (wd & 7);
    }
    uint64_t fcs = 0;
    for (int i = 0; i < fcs_bytes; i++) fcs |= (uint64_t)src[p + i] << (8 * i);
    if (fcs_bytes == 2) fcs += 256;
    p += fcs_bytes;
    if (single) window = fcs;
    const uint32_t bsz = (uint32_t)(window < BLOCK_MAX ? window : BLOCK_MAX);
    uint64_t o = 0, tbl = 0;
    uint32_t tbl_len = 0, n = 0, nseq = 0;
    for (;;) {
        if (len - p < 3) return false;
        const uint64_t hdr = p;
        const uint32_t bh = rd24(src + p);
        p += 3;
        const int last = bh & 1, type = (bh >> 1) & 3;
        const uint32_t bsize = bh >> 3;
        if (type == 3 || bsize > BLOCK_MAX || (type == 2 && bsize == BLOCK_MAX)) return false;
        uint64_t bout;
        uint32_t dlen = 0;
        bool seq = false;
        if (type == 0) {
            if (len - p < bsize) return false;
            bout = bsize;
        } else if (type == 1) {
            if (len - p < 1) return false;
            bout = bsize;
        } else {
            if (len - p < bsize) return false;
            const uint8_t *b = src + p;
            LitHdr h;
            if (!lit_header(b, bsize, &h)) return false;
            seq = h.lsec + 1 != bsize || b[h.lsec] != 0;
            if (h.ltype == 2) {
                tbl = p + h.hs;
                tbl_len = huf_desc_bytes(b[h.hs]);
                if (tbl_len > h.csize) return false;
            } else if (h.ltype == 3 && tbl_len == 0) {
                return false;  // treeless without an earlier description
            }
            if (h.ltype >= 2) dlen = tbl_len;
            bout = h.regen;
            if (seq) {  // one block size; the last block the rest of the content
                if (last && !fcs_bytes) return false;
                bout = last ? (fcs >= o ? fcs - o : 0) : bsz;
                if (bout < h.regen || bout > BLOCK_MAX) return false;
                nseq++;
            }
        }
        if (o + bout > cap) return false;
        if (d) {
            BlockDesc &e = d[n];
            e.src = p;
            e.out = o;
            e.tbl = dlen ? tbl : 0;
            e.job = job;
            e.meta = bsize | ((uint32_t)type << 18) | (dlen << 20) | (seq ? META_SEQ : 0);
            e.slot = ~0u;
            e.pad = 0;
        }
        n++;
        o += bout;
        p += type == 1 ? 1 : bsize;
        if (last) {
            jp->lastpos = hdr;
            break;
        }
    }
    if (fcs_bytes && o != fcs) return false;
    jp->ckpos = ~0ull;
    if (cksum) {
        if (len - p < 4) return false;
        jp->ckpos = p;
        p += 4;
    }
    if (p != len) return false;  // one frame per job
    jp->total = o;
    jp->count = n;
    jp->nseq = nseq;
    jp->bsz = bsz;
    *count = n;
    return true;
}

// One block without sequences of a block-parallel frame into dst (the
// job's output).  False when it does not decode.  All lanes.
template <class W>
ZHD bool decode_block(W *ws, const uint8_t *src, const BlockDesc &e, uint8_t *dst, int lane, int nl) {
    const uint32_t bsize = e.meta & 0x3FFFF, type = (e.meta >> 18) & 3, dlen = (e.meta >> 20) & 0xFF;
    const uint8_t *b = src + e.src;
    uint8_t *out = dst + e.out;
    if (type == 0) {
        coop_copy(out, b, bsize, lane, nl);
        return true;
    }
    if (type == 1) {
        coop_fill(out, b[0], bsize, lane, nl);
        return true;
    }
    LitHdr h;
    if (!lit_header(b, bsize, &h)) return false;
    if (h.ltype == 0) {
        coop_copy(out, b + h.hs, h.regen, lane, nl);
        return true;
    }
    if (h.ltype == 1) {
        coop_fill(out, b[h.hs], h.regen, lane, nl);
        return true;
    }
    if (lane == 0)
        ws->err = huf_read_table(ws, src + e.tbl, dlen) == (int)dlen && ws->huf_log <= W::TAB_LOG
                      ? OK
                      : E_CORRUPT;
    warp_sync();
    if (ws->err) return false;
    huf_fill(ws, lane, nl);
    warp_sync();
    const uint8_t *p = b + h.hs + (h.ltype == 2 ? dlen : 0);
    return lit_streams(ws, p, b + h.hs + h.csize, h.nstreams, h.regen, out, lane, nl);
}

// The blocks with sequences of a block-parallel job, in order, after every
// other block is in place (matches read earlier blocks' output): the serial
// block decoder with the frame's repeat offsets and sequence tables carried
// from one to the next.  False when one fails or regenerates another size
// than planned.  All lanes.
ZHD bool decode_seq_blocks(Workspace *ws, const Job &job, const JobPlan &jp, const BlockDesc *d,
                           const uint8_t *slots, int lane, int nl) {
    if (lane == 0) {
        ws->rep[0] = 1;
        ws->rep[1] = 4;
        ws->rep[2] = 8;
        ws->ll_log = ws->ml_log = ws->of_log = ws->huf_log = -1;
    }
    warp_sync();
    uint64_t built = ~0ull;  // description the Huffman table holds
    for (uint32_t i = 0; i < jp.count; i++) {
        const BlockDesc e = d[i];
        if (!(e.meta & META_SEQ)) continue;
        const uint32_t bsize = e.meta & 0x3FFFF, dlen = (e.meta >> 20) & 0xFF;
        const uint8_t *b = job.src + e.src;
        const uint8_t *pre = (b[0] & 3) >= 2 && e.slot != ~0u ? slots + (uint64_t)e.slot * LIT_SCRATCH : nullptr;
        if (!pre && (b[0] & 3) == 3 && built != e.tbl) {  // treeless: the last description's table
            if (lane == 0) ws->err = huf_read_table(ws, job.src + e.tbl, dlen) == (int)dlen ? OK : E_CORRUPT;
            warp_sync();
            if (ws->err) return false;
            huf_fill(ws, lane, nl);
            warp_sync();
        }
        if (!pre && (b[0] & 3) >= 2) built = e.tbl;
        uint64_t o = e.out;
        if (decode_compressed_block(ws, job, b, bsize, 0, &o, lane, nl, pre) != OK) return false;
        const uint64_t want = (i + 1 == jp.count) ? jp.total - e.out : jp.bsz;
        if (o - e.out != want) return false;
    }
    return true;
}

}  // namespace zs
}  // namespace hct
