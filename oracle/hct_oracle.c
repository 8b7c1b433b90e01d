/*
 * hct_oracle.c -- CPU restatement of the reference's HCT decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: tests/, the
 * smoke check and bench.py's CPU-baseline leg may call it, the product path
 * never does.  Every function cites the reference source it restates
 * (paths relative to the haagenti repository root).
 *
 *   LZ4 block codec ........ crates/haagenti-lz4/src/block.rs:12-373
 *   INT4 codec ............. crates/haagenti/src/testing/quantization.rs:30-210
 *   DCT-II / DCT-III ....... crates/haagenti-core/src/dct.rs:79-337
 *   spectral top-k bitmap .. crates/haagenti/src/compressive.rs:140-172
 *
 * The FFT under the Makhoul DCT is our own mixed-radix decimation-in-time
 * FFT; the reference uses rustfft 6.4.1, whose exact f32 rounding is not
 * reproduced (the IDCT is checked against an f64 truth with a tolerance).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Status codes shared with the CUDA library (include/hct_b200.h); each maps
 * 1:1 to a haagenti_core::Error variant raised by block.rs. */
enum {
    ORC_OK = 0,
    ORC_UNEXPECTED_EOF = 1,   /* Error::UnexpectedEof{bytes_read}          */
    ORC_BUFFER_TOO_SMALL = 2, /* Error::BufferTooSmall{required,provided}  */
    ORC_ZERO_OFFSET = 3,      /* Error::corrupted("invalid zero offset")   */
    ORC_OFFSET_BEYOND = 4     /* Error::corrupted_at("offset beyond output", pos) */
};

/* ======================================================================
 * LZ4 block format (block.rs)
 * ====================================================================== */

#define LZ4_MIN_MATCH 4u          /* block.rs:15 */
#define LZ4_HASH_TABLE_SIZE 65536u /* block.rs:21 */
#define LZ4_ACCELERATION 1u       /* block.rs:24 */
#define LZ4_LAST_LITERALS 5u      /* block.rs:27 */
#define LZ4_MIN_INPUT_SIZE 13u    /* block.rs:30 */

static inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* block.rs:34-37 */
static inline size_t lz4_hash(uint32_t v) {
    return (size_t)((v * 2654435761u) >> 16) & (LZ4_HASH_TABLE_SIZE - 1);
}

/* block.rs:370-373 */
size_t orc_lz4_max_compressed_size(size_t n) { return n + n / 255 + 16; }

/* block.rs:212-251: token, literal-length extension, literals. */
static int write_last_literals(const uint8_t *in, uint8_t *out, size_t cap, size_t *pos_io,
                               size_t lit_start, size_t lit_len, size_t *req) {
    size_t pos = *pos_io;
    size_t needed = 1 + lit_len / 255 + 1 + lit_len;
    if (pos + needed > cap) {
        *req = pos + needed;
        return ORC_BUFFER_TOO_SMALL;
    }
    size_t ll = lit_len < 15 ? lit_len : 15;
    out[pos++] = (uint8_t)(ll << 4);
    if (lit_len >= 15) {
        size_t rem = lit_len - 15;
        while (rem >= 255) { out[pos++] = 255; rem -= 255; }
        out[pos++] = (uint8_t)rem;
    }
    memcpy(out + pos, in + lit_start, lit_len);
    pos += lit_len;
    *pos_io = pos;
    return ORC_OK;
}

/* block.rs:150-209 */
static int write_sequence(const uint8_t *in, uint8_t *out, size_t cap, size_t *pos_io,
                          size_t lit_start, size_t lit_len, uint16_t offset, size_t match_len,
                          size_t *req) {
    size_t pos = *pos_io;
    size_t ll = lit_len < 15 ? lit_len : 15;
    size_t ml = (match_len - LZ4_MIN_MATCH) < 15 ? (match_len - LZ4_MIN_MATCH) : 15;
    uint8_t token = (uint8_t)((ll << 4) | ml);
    size_t needed = 1 + lit_len / 255 + 1 + lit_len + 2 + (match_len - LZ4_MIN_MATCH) / 255 + 1;
    if (pos + needed > cap) {
        *req = pos + needed;
        return ORC_BUFFER_TOO_SMALL;
    }
    out[pos++] = token;
    if (lit_len >= 15) {
        size_t rem = lit_len - 15;
        while (rem >= 255) { out[pos++] = 255; rem -= 255; }
        out[pos++] = (uint8_t)rem;
    }
    memcpy(out + pos, in + lit_start, lit_len);
    pos += lit_len;
    out[pos++] = (uint8_t)(offset & 0xff);
    out[pos++] = (uint8_t)(offset >> 8);
    if (match_len - LZ4_MIN_MATCH >= 15) {
        size_t rem = match_len - LZ4_MIN_MATCH - 15;
        while (rem >= 255) { out[pos++] = 255; rem -= 255; }
        out[pos++] = (uint8_t)rem;
    }
    *pos_io = pos;
    return ORC_OK;
}

/*
 * block.rs:73-147, greedy LZ4 with a 64 Ki-entry hash table.
 * The reference zero-fills a fresh table per call; a generation tag per
 * entry gives the same lookups ("never written" reads as position 0)
 * without clearing 512 KiB per 16 KiB block.
 */
typedef struct { uint32_t pos; uint32_t gen; } hslot;
static _Thread_local hslot *tl_table = NULL;
static _Thread_local uint32_t tl_gen = 0;

int orc_lz4_compress_block(const uint8_t *in, size_t n, uint8_t *out, size_t cap,
                           size_t *out_len, size_t *req) {
    size_t pos = 0;
    *req = 0;
    if (n < LZ4_MIN_INPUT_SIZE) {
        int rc = write_last_literals(in, out, cap, &pos, 0, n, req);
        *out_len = pos;
        return rc;
    }
    if (!tl_table) {
        tl_table = (hslot *)calloc(LZ4_HASH_TABLE_SIZE, sizeof(hslot));
        tl_gen = 0;
    }
    tl_gen++;
    if (tl_gen == 0) { /* wrapped: clear once */
        memset(tl_table, 0, LZ4_HASH_TABLE_SIZE * sizeof(hslot));
        tl_gen = 1;
    }
    const uint32_t gen = tl_gen;
    size_t input_pos = 0, anchor = 0;
    size_t match_limit = n > LZ4_LAST_LITERALS ? n - LZ4_LAST_LITERALS : 0;
    size_t mf_limit = match_limit > LZ4_MIN_MATCH ? match_limit - LZ4_MIN_MATCH : 0;

    while (input_pos < mf_limit) {
        size_t h = lz4_hash(rd32(in + input_pos));
        size_t match_pos = tl_table[h].gen == gen ? tl_table[h].pos : 0;
        tl_table[h].pos = (uint32_t)input_pos;
        tl_table[h].gen = gen;
        if (match_pos > 0 && input_pos - match_pos <= 65535 &&
            rd32(in + match_pos) == rd32(in + input_pos)) {
            /* count_match, block.rs:61-68 */
            size_t p1 = match_pos + LZ4_MIN_MATCH, p2 = input_pos + LZ4_MIN_MATCH, start = p2;
            while (p2 < match_limit && in[p1] == in[p2]) { p1++; p2++; }
            size_t match_len = LZ4_MIN_MATCH + (p2 - start);
            size_t lit_len = input_pos - anchor;
            uint16_t offset = (uint16_t)(input_pos - match_pos);
            int rc = write_sequence(in, out, cap, &pos, anchor, lit_len, offset, match_len, req);
            if (rc) { *out_len = pos; return rc; }
            input_pos += match_len;
            anchor = input_pos;
            if (input_pos < mf_limit) {
                size_t h2 = lz4_hash(rd32(in + input_pos - 2));
                tl_table[h2].pos = (uint32_t)(input_pos - 2);
                tl_table[h2].gen = gen;
            }
        } else {
            input_pos += LZ4_ACCELERATION;
        }
    }
    size_t lit_len = n - anchor;
    if (lit_len > 0) {
        int rc = write_last_literals(in, out, cap, &pos, anchor, lit_len, req);
        if (rc) { *out_len = pos; return rc; }
    }
    *out_len = pos;
    return ORC_OK;
}

/*
 * block.rs:261-366.  `cap` is output.len(), `output_size` the expected size
 * that ends the token loop after a literal run.  On error, *pos_out holds the
 * value the reference reports (bytes_read for EOF, output_pos for the
 * offset error, `required` for BufferTooSmall) and *aux the `provided` size.
 */
int orc_lz4_decompress_block(const uint8_t *in, size_t in_len, uint8_t *out, size_t cap,
                             size_t output_size, size_t *written, size_t *pos_out, size_t *aux) {
    size_t ip = 0, op = 0;
    *pos_out = 0;
    *aux = 0;
    while (ip < in_len) {
        uint8_t token = in[ip++];
        size_t lit = token >> 4;
        size_t ml = token & 0x0f;
        if (lit == 15) {
            for (;;) {
                if (ip >= in_len) { *pos_out = ip; *written = op; return ORC_UNEXPECTED_EOF; }
                uint8_t b = in[ip++];
                lit += b;
                if (b != 255) break;
            }
        }
        if (lit > 0) {
            if (ip + lit > in_len) { *pos_out = ip; *written = op; return ORC_UNEXPECTED_EOF; }
            if (op + lit > cap) { *pos_out = op + lit; *aux = cap; *written = op; return ORC_BUFFER_TOO_SMALL; }
            memcpy(out + op, in + ip, lit);
            ip += lit;
            op += lit;
        }
        if (op >= output_size) break;
        if (ip + 2 > in_len) { *pos_out = ip; *written = op; return ORC_UNEXPECTED_EOF; }
        size_t offset = (size_t)in[ip] | ((size_t)in[ip + 1] << 8);
        ip += 2;
        if (offset == 0) { *pos_out = op; *written = op; return ORC_ZERO_OFFSET; }
        if (offset > op) { *pos_out = op; *written = op; return ORC_OFFSET_BEYOND; }
        ml += LZ4_MIN_MATCH;
        if ((token & 0x0f) == 15) {
            for (;;) {
                if (ip >= in_len) { *pos_out = ip; *written = op; return ORC_UNEXPECTED_EOF; }
                uint8_t b = in[ip++];
                ml += b;
                if (b != 255) break;
            }
        }
        size_t ms = op - offset;
        if (op + ml > cap) { *pos_out = op + ml; *aux = cap; *written = op; return ORC_BUFFER_TOO_SMALL; }
        if (offset >= ml) {
            memmove(out + op, out + ms, ml);
        } else {
            for (size_t i = 0; i < ml; i++) out[op + i] = out[ms + i];
        }
        op += ml;
    }
    *written = op;
    return ORC_OK;
}

/* Batch helpers (many independent blocks, one OpenMP thread per block). */
typedef struct {
    uint64_t src_off, dst_off;
    uint32_t src_len, dst_cap, out_size, pad;
} orc_block_desc;

typedef struct {
    int32_t code, pad;
    uint64_t position, aux, written;
} orc_block_status;

void orc_lz4_decompress_batch(const uint8_t *src, const orc_block_desc *d, size_t nblocks,
                              uint8_t *dst, orc_block_status *st, int threads) {
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
    for (long i = 0; i < (long)nblocks; i++) {
        size_t w = 0, p = 0, a = 0;
        int rc = orc_lz4_decompress_block(src + d[i].src_off, d[i].src_len, dst + d[i].dst_off,
                                          d[i].dst_cap, d[i].out_size, &w, &p, &a);
        st[i].code = rc;
        st[i].position = p;
        st[i].aux = a;
        st[i].written = w;
    }
}

/* Compress `n` bytes in `block` sized chunks (HctWriter::compress_data,
 * tensor.rs:556-562 with Lz4Compressor::compress, compress.rs:60-99).
 * Block i lands at out + i*out_stride, its length in lens[i]. */
int orc_lz4_compress_chunks(const uint8_t *in, size_t n, size_t block, uint8_t *out,
                            size_t out_stride, uint32_t *lens, int threads) {
    size_t nb = n == 0 ? 0 : (n + block - 1) / block;
    int bad = 0;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 8) reduction(| : bad)
#endif
    for (long i = 0; i < (long)nb; i++) {
        size_t s = (size_t)i * block;
        size_t len = (n - s) < block ? (n - s) : block;
        size_t ol = 0, req = 0;
        int rc = orc_lz4_compress_block(in + s, len, out + (size_t)i * out_stride, out_stride, &ol, &req);
        lens[i] = (uint32_t)ol;
        bad |= rc;
    }
    return bad;
}

/* ======================================================================
 * INT4 codec (testing/quantization.rs)
 * ====================================================================== */

#define Q4_BLOCK 32u /* quantization.rs:10 */

/* quantization.rs:136-163: truncating, flush-to-zero f32 -> f16. */
uint16_t orc_f32_to_f16_bits(float val) {
    uint32_t bits;
    memcpy(&bits, &val, 4);
    uint32_t sign = (bits >> 31) & 1;
    int32_t exp = (int32_t)((bits >> 23) & 0xff);
    uint32_t frac = bits & 0x7fffff;
    if (exp == 0) return (uint16_t)(sign << 15);
    if (exp == 0xff) return (uint16_t)((sign << 15) | (0x1f << 10) | (frac >> 13));
    int32_t ne = exp - 127 + 15;
    if (ne >= 31) return (uint16_t)((sign << 15) | (0x1f << 10));
    if (ne <= 0) return (uint16_t)(sign << 15);
    return (uint16_t)((sign << 15) | ((uint32_t)ne << 10) | (frac >> 13));
}

/* quantization.rs:166-197: exact f16 -> f32 (subnormals normalised). */
float orc_f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (h >> 15) & 1, exp = (h >> 10) & 0x1f, frac = h & 0x3ff, out;
    if (exp == 0) {
        if (frac == 0) {
            out = sign << 31;
        } else {
            int32_t e = -14;
            uint32_t f = frac;
            while ((f & 0x400) == 0) { f <<= 1; e -= 1; }
            f &= 0x3ff;
            out = (sign << 31) | ((uint32_t)((e + 127) & 0xff) << 23) | (f << 13);
        }
    } else if (exp == 31) {
        out = (sign << 31) | (0xffu << 23) | (frac << 13);
    } else {
        out = (sign << 31) | ((exp - 15 + 127) << 23) | (frac << 13);
    }
    float r;
    memcpy(&r, &out, 4);
    return r;
}

/* quantization.rs:202-210 */
size_t orc_int4_compressed_size(size_t n) {
    if (n == 0) return 0;
    return ((n + Q4_BLOCK - 1) / Q4_BLOCK) * 2 + (n + 1) / 2;
}

/* Rust `f32::round() as i8`: half away from zero, saturating, NaN -> 0. */
static inline int rust_round_i8(float x) {
    float r = roundf(x);
    if (r != r) return 0;
    if (r < -128.0f) return -128;
    if (r > 127.0f) return 127;
    return (int)r;
}

/* quantization.rs:30-70.  `out` must hold orc_int4_compressed_size(n). */
void orc_quantize_int4(const float *w, size_t n, uint8_t *out) {
    if (n == 0) return;
    size_t nb = (n + Q4_BLOCK - 1) / Q4_BLOCK;
    uint8_t *nib = out + nb * 2;
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * Q4_BLOCK, e = s + Q4_BLOCK < n ? s + Q4_BLOCK : n;
        float max_abs = 0.0f;
        for (size_t i = s; i < e; i++) max_abs = fmaxf(max_abs, fabsf(w[i]));
        float scale = max_abs > 1e-10f ? max_abs / 7.0f : 1.0f;
        uint16_t h = orc_f32_to_f16_bits(scale);
        out[2 * b] = (uint8_t)(h & 0xff);
        out[2 * b + 1] = (uint8_t)(h >> 8);
        for (size_t i = s; i < e; i++) {
            int q = rust_round_i8(w[i] / scale);
            if (q < -8) q = -8;
            if (q > 7) q = 7;
            uint8_t v = (uint8_t)(q + 8);
            if (i & 1) nib[i >> 1] |= (uint8_t)((v & 0x0f) << 4);
            else nib[i >> 1] = (uint8_t)(v & 0x0f);
        }
    }
}

/* quantization.rs:82-131.  Returns the number of elements written
 * (0 when the scales do not fit, fewer than n when the nibbles run out). */
size_t orc_dequantize_int4(const uint8_t *data, size_t len, size_t n, float *out) {
    if (n == 0) return 0;
    size_t nb = (n + Q4_BLOCK - 1) / Q4_BLOCK;
    size_t sb = nb * 2;
    if (len < sb) return 0;
    const uint8_t *packed = data + sb;
    size_t plen = len - sb;
    size_t w = 0;
    for (size_t b = 0; b < nb; b++) {
        float scale = orc_f16_bits_to_f32((uint16_t)(data[2 * b] | (data[2 * b + 1] << 8)));
        size_t bs = n - b * Q4_BLOCK < Q4_BLOCK ? n - b * Q4_BLOCK : Q4_BLOCK;
        for (size_t j = 0; j < bs; j++) {
            size_t byte = w >> 1;
            if (byte >= plen) return w;
            uint8_t nibble = (w & 1) ? (packed[byte] >> 4) & 0x0f : packed[byte] & 0x0f;
            int8_t q = (int8_t)nibble - 8;
            out[w] = (float)q * scale;
            w++;
        }
    }
    return w;
}

/* orc_dequantize_int4 split over OpenMP threads, 32-element block by block:
 * each element is the same f32 product; written = min(n, 2 * nibble bytes)
 * (0 when the scales do not fit), as the serial loop stops. */
size_t orc_dequantize_int4_threads(const uint8_t *data, size_t len, size_t n, float *out,
                                   int threads) {
    if (n == 0) return 0;
    size_t nb = (n + Q4_BLOCK - 1) / Q4_BLOCK;
    size_t sb = nb * 2;
    if (len < sb) return 0;
    const uint8_t *packed = data + sb;
    size_t plen = len - sb;
    size_t w = 2 * plen < n ? 2 * plen : n;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
    for (long long b = 0; b < (long long)nb; b++) {
        float scale = orc_f16_bits_to_f32((uint16_t)(data[2 * b] | (data[2 * b + 1] << 8)));
        size_t s = (size_t)b * Q4_BLOCK, e = s + Q4_BLOCK < w ? s + Q4_BLOCK : w;
        for (size_t i = s; i < e; i++) {
            uint8_t nibble = (i & 1) ? (packed[i >> 1] >> 4) & 0x0f : packed[i >> 1] & 0x0f;
            out[i] = (float)((int8_t)nibble - 8) * scale;
        }
    }
    return w;
}

/* f32 -> f16 with IEEE round-to-nearest-even, subnormals and overflow to
 * infinity: the conversion of half 2.7.1's f16::from_f32 that
 * mixed_precision.rs:463 stores its scales with (infinity and NaN map to
 * the f16 infinity / a quiet NaN). */
uint16_t orc_f32_to_f16_rne(float val) {
    uint32_t bits;
    memcpy(&bits, &val, 4);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const int32_t exp = (int32_t)((bits >> 23) & 0xff);
    const uint32_t mant = bits & 0x7fffffu;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (mant ? 0x200u : 0u));
    const int32_t e = exp - 127;
    if (e > 15) return (uint16_t)(sign | 0x7c00u);
    if (e >= -14) {  /* normal half: keep 10 mantissa bits, round the other 13 */
        uint32_t h = ((uint32_t)(e + 15) << 10) | (mant >> 13);
        const uint32_t rest = mant & 0x1fffu;
        if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) h++;  /* may carry to inf */
        return (uint16_t)(sign | h);
    }
    if (exp == 0) return (uint16_t)sign;  /* f32 zero or subnormal: far below 2^-25 */
    /* subnormal half: units of 2^-24; value = m * 2^(e-23), m with the implicit 1 */
    const uint32_t m = mant | 0x800000u;
    const int32_t sh = -(e + 1); /* >= 14 */
    if (sh > 24) return (uint16_t)sign;
    uint32_t h = m >> sh;
    const uint32_t rest = m & ((1u << sh) - 1u), halfway = 1u << (sh - 1);
    if (rest > halfway || (rest == halfway && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

/* mixed_precision.rs:448-486: the quantize_int4 of quantization.rs:30-70
 * with the scale stored as the round-to-nearest-even f16.  `out` must hold
 * orc_int4_compressed_size(n). */
void orc_quantize_int4_mp(const float *w, size_t n, uint8_t *out) {
    if (n == 0) return;
    size_t nb = (n + Q4_BLOCK - 1) / Q4_BLOCK;
    uint8_t *nib = out + nb * 2;
    for (size_t b = 0; b < nb; b++) {
        size_t s = b * Q4_BLOCK, e = s + Q4_BLOCK < n ? s + Q4_BLOCK : n;
        float max_abs = 0.0f;
        for (size_t i = s; i < e; i++) max_abs = fmaxf(max_abs, fabsf(w[i]));
        float scale = max_abs > 1e-10f ? max_abs / 7.0f : 1.0f;
        uint16_t h = orc_f32_to_f16_rne(scale);
        out[2 * b] = (uint8_t)(h & 0xff);
        out[2 * b + 1] = (uint8_t)(h >> 8);
        for (size_t i = s; i < e; i++) {
            int q = rust_round_i8(w[i] / scale);
            if (q < -8) q = -8;
            if (q > 7) q = 7;
            uint8_t v = (uint8_t)(q + 8);
            if (i & 1) nib[i >> 1] |= (uint8_t)((v & 0x0f) << 4);
            else nib[i >> 1] = (uint8_t)(v & 0x0f);
        }
    }
}

/* mixed_precision.rs:489-539.  Returns the number of values written: 0 for
 * n == 0 or empty data, else n -- all zero when the scales do not fit,
 * zero past the end of the nibbles. */
size_t orc_dequantize_int4_mp(const uint8_t *data, size_t len, size_t n, float *out) {
    if (n == 0 || len == 0) return 0;
    size_t nb = (n + Q4_BLOCK - 1) / Q4_BLOCK;
    size_t sb = nb * 2;
    if (len < sb) {
        for (size_t i = 0; i < n; i++) out[i] = 0.0f;
        return n;
    }
    const uint8_t *packed = data + sb;
    size_t plen = len - sb;
    for (size_t i = 0; i < n; i++) {
        size_t b = i / Q4_BLOCK, byte = i >> 1;
        if (byte >= plen) { out[i] = 0.0f; continue; }
        float scale = orc_f16_bits_to_f32((uint16_t)(data[2 * b] | (data[2 * b + 1] << 8)));
        uint8_t nibble = (i & 1) ? (packed[byte] >> 4) & 0x0f : packed[byte] & 0x0f;
        out[i] = (float)((int8_t)nibble - 8) * scale;
    }
    return n;
}

/* ======================================================================
 * Mixed-radix complex FFT (f32 data, twiddles rounded from f64)
 * ====================================================================== */

typedef struct { float re, im; } cpx;

typedef struct {
    size_t n;
    int inverse;
    int nf;
    size_t fac[64];  /* radices, outermost first */
    cpx *tw;         /* tw[j] = exp(-+2 pi i j / n), j < n */
} fft_plan;

static void plan_init(fft_plan *p, size_t n, int inverse) {
    p->n = n;
    p->inverse = inverse;
    p->nf = 0;
    size_t m = n;
    static const size_t pref[] = {4, 2, 3, 5, 7};
    for (int i = 0; i < 5 && m > 1; i++) {
        while (m % pref[i] == 0) { p->fac[p->nf++] = pref[i]; m /= pref[i]; }
    }
    for (size_t f = 11; m > 1; f += 2) {
        while (m % f == 0) { p->fac[p->nf++] = f; m /= f; }
        if (f * f > m && m > 1) { p->fac[p->nf++] = m; m = 1; }
    }
    p->tw = (cpx *)malloc(sizeof(cpx) * (n ? n : 1));
    double sgn = inverse ? 1.0 : -1.0;
    for (size_t j = 0; j < n; j++) {
        double a = sgn * 2.0 * M_PI * (double)j / (double)n;
        p->tw[j].re = (float)cos(a);
        p->tw[j].im = (float)sin(a);
    }
}

static void plan_free(fft_plan *p) { free(p->tw); }

static inline cpx cmul(cpx a, cpx b) {
    cpx r = {a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re};
    return r;
}

/* out[k*ostride] for k < n  <-  DFT of in[j*istride], j < n; n = prod fac[lvl..]. */
static void fft_rec(const fft_plan *p, const cpx *in, size_t istride, cpx *out, size_t n,
                    int lvl, size_t twstep, cpx *scratch) {
    if (n == 1) { out[0] = in[0]; return; }
    size_t r = p->fac[lvl], m = n / r;
    /* r sub-transforms of length m on the decimated inputs, stored contiguously */
    for (size_t q = 0; q < r; q++)
        fft_rec(p, in + q * istride, istride * r, out + q * m, m, lvl + 1, twstep * r, scratch);
    /* butterflies: X[k + s*m] = sum_q W_n^{q(k+s m)} Y_q[k] */
    for (size_t k = 0; k < m; k++) {
        cpx *y = scratch;
        for (size_t q = 0; q < r; q++) {
            cpx v = out[q * m + k];
            y[q] = q ? cmul(v, p->tw[(q * k * twstep) % p->n]) : v;
        }
        if (r == 2) {
            cpx a = y[0], b = y[1];
            out[k].re = a.re + b.re; out[k].im = a.im + b.im;
            out[k + m].re = a.re - b.re; out[k + m].im = a.im - b.im;
        } else if (r == 4) {
            cpx a = y[0], b = y[1], c = y[2], d = y[3];
            cpx s0 = {a.re + c.re, a.im + c.im}, s1 = {a.re - c.re, a.im - c.im};
            cpx s2 = {b.re + d.re, b.im + d.im}, s3 = {b.re - d.re, b.im - d.im};
            /* multiply s3 by -i (forward) or +i (inverse) */
            cpx s3r = p->inverse ? (cpx){-s3.im, s3.re} : (cpx){s3.im, -s3.re};
            out[k].re = s0.re + s2.re; out[k].im = s0.im + s2.im;
            out[k + m].re = s1.re + s3r.re; out[k + m].im = s1.im + s3r.im;
            out[k + 2 * m].re = s0.re - s2.re; out[k + 2 * m].im = s0.im - s2.im;
            out[k + 3 * m].re = s1.re - s3r.re; out[k + 3 * m].im = s1.im - s3r.im;
        } else {
            for (size_t s = 0; s < r; s++) {
                cpx acc = {0.0f, 0.0f};
                for (size_t q = 0; q < r; q++) {
                    cpx w = p->tw[((q * s) % r) * (p->n / r)];
                    cpx t = cmul(y[q], w);
                    acc.re += t.re; acc.im += t.im;
                }
                out[k + s * m] = acc;
            }
        }
    }
}

static void fft_exec(const fft_plan *p, const cpx *in, cpx *out) {
    cpx scratch[256];
    cpx *sc = scratch;
    size_t maxr = 0;
    for (int i = 0; i < p->nf; i++) if (p->fac[i] > maxr) maxr = p->fac[i];
    if (maxr > 256) sc = (cpx *)malloc(sizeof(cpx) * maxr);
    fft_rec(p, in, 1, out, p->n, 0, 1, sc);
    if (sc != scratch) free(sc);
}

/* ======================================================================
 * DCT (dct.rs)
 * ====================================================================== */

/* dct.rs:133-146 */
static void dct_1d_direct(const float *in, float *out, size_t n) {
    float scale = sqrtf(2.0f / (float)n);
    for (size_t k = 0; k < n; k++) {
        float sum = 0.0f;
        for (size_t i = 0; i < n; i++)
            sum += in[i] * cosf((float)M_PI * (float)k * ((float)i + 0.5f) / (float)n);
        out[k] = sum * scale;
    }
    out[0] /= (float)M_SQRT2;
}

/* dct.rs:263-277 */
static void idct_1d_direct(const float *in, float *out, size_t n) {
    float scale = sqrtf(2.0f / (float)n);
    for (size_t i = 0; i < n; i++) {
        float sum = in[0] / (float)M_SQRT2;
        for (size_t k = 1; k < n; k++)
            sum += in[k] * cosf((float)M_PI * (float)k * ((float)i + 0.5f) / (float)n);
        out[i] = sum * scale;
    }
}

typedef struct {
    size_t n;
    fft_plan fwd, inv;
    cpx *y, *z;
} dct_ws;

static void ws_init(dct_ws *w, size_t n) {
    w->n = n;
    if (n > 32) {
        plan_init(&w->fwd, n, 0);
        plan_init(&w->inv, n, 1);
    }
    w->y = (cpx *)malloc(sizeof(cpx) * n);
    w->z = (cpx *)malloc(sizeof(cpx) * n);
}

static void ws_free(dct_ws *w) {
    if (w->n > 32) { plan_free(&w->fwd); plan_free(&w->inv); }
    free(w->y);
    free(w->z);
}

/* dct.rs:79-129, Makhoul DCT-II */
static void dct_1d_ws(dct_ws *w, const float *in, float *out) {
    size_t n = w->n;
    if (n == 0) return;
    if (n <= 32) { dct_1d_direct(in, out, n); return; }
    cpx *y = w->y, *Y = w->z;
    for (size_t k = 0; k < n; k++) { y[k].re = 0.0f; y[k].im = 0.0f; }
    for (size_t k = 0; k < (n + 1) / 2; k++) if (2 * k < n) y[k].re = in[2 * k];
    for (size_t k = 0; k < n / 2; k++) if (2 * k + 1 < n) y[n - 1 - k].re = in[2 * k + 1];
    fft_exec(&w->fwd, y, Y);
    float scale = sqrtf(2.0f / (float)n);
    for (size_t k = 0; k < n; k++) {
        float angle = -(float)M_PI * (float)k / (2.0f * (float)n);
        cpx tw = {cosf(angle), sinf(angle)};
        out[k] = cmul(Y[k], tw).re * scale;
    }
    out[0] /= (float)M_SQRT2;
}

/* dct.rs:154-259, inverse Makhoul DCT-III */
static void idct_1d_ws(dct_ws *w, const float *in, float *out) {
    size_t n = w->n;
    if (n == 0) return;
    if (n <= 32) { idct_1d_direct(in, out, n); return; }
    cpx *y = w->y, *v = w->z;
    float scale = sqrtf(2.0f / (float)n);
    /* c[k] is used in place of the reference's scratch vector */
    float c0 = in[0] * (float)M_SQRT2 / scale;
    for (size_t k = 0; k < n; k++) { y[k].re = 0.0f; y[k].im = 0.0f; }
    y[0].re = c0;
    if (n % 2 == 0) {
        size_t k = n / 2;
        float angle = -(float)M_PI * (float)k / (2.0f * (float)n);
        y[k].re = (in[k] / scale) / cosf(angle);
        y[k].im = 0.0f;
    }
    size_t limit = (n % 2 == 0) ? n / 2 : (n + 1) / 2;
    for (size_t k = 1; k < limit; k++) {
        float ak = -(float)M_PI * (float)k / (2.0f * (float)n);
        float ank = -(float)M_PI * (float)(n - k) / (2.0f * (float)n);
        float ck = cosf(ak), sk = sinf(ak), cnk = cosf(ank), snk = sinf(ank);
        float Ck = in[k] / scale, Cnk = in[n - k] / scale;
        float det = ck * snk + sk * cnk;
        float yr = (Ck * snk + Cnk * sk) / det;
        float yi = (Cnk * ck - Ck * cnk) / det;
        y[k].re = yr; y[k].im = yi;
        y[n - k].re = yr; y[n - k].im = -yi;
    }
    fft_exec(&w->inv, y, v);
    float inv_n = 1.0f / (float)n;
    for (size_t k = 0; k < (n + 1) / 2; k++) if (2 * k < n) out[2 * k] = v[k].re * inv_n;
    for (size_t k = 0; k < n / 2; k++) if (2 * k + 1 < n) out[2 * k + 1] = v[n - 1 - k].re * inv_n;
}

void orc_dct_1d(const float *in, float *out, size_t n) {
    dct_ws w; ws_init(&w, n); dct_1d_ws(&w, in, out); ws_free(&w);
}

void orc_idct_1d(const float *in, float *out, size_t n) {
    dct_ws w; ws_init(&w, n); idct_1d_ws(&w, in, out); ws_free(&w);
}

/* dct.rs:282-308: rows first, then columns.  Threaded over rows/columns. */
void orc_dct_2d(const float *in, float *out, size_t width, size_t height, int threads) {
    float *temp = (float *)malloc(sizeof(float) * width * height);
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        dct_ws wr; ws_init(&wr, width);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long y = 0; y < (long)height; y++) dct_1d_ws(&wr, in + y * width, temp + y * width);
        ws_free(&wr);
        dct_ws wc; ws_init(&wc, height);
        float *cb = (float *)malloc(sizeof(float) * height), *co = (float *)malloc(sizeof(float) * height);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long x = 0; x < (long)width; x++) {
            for (size_t y = 0; y < height; y++) cb[y] = temp[y * width + x];
            dct_1d_ws(&wc, cb, co);
            for (size_t y = 0; y < height; y++) out[y * width + x] = co[y];
        }
        free(cb); free(co); ws_free(&wc);
    }
    free(temp);
}

/* dct.rs:311-337: columns first, then rows. */
void orc_idct_2d(const float *in, float *out, size_t width, size_t height, int threads) {
    float *temp = (float *)malloc(sizeof(float) * width * height);
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        dct_ws wc; ws_init(&wc, height);
        float *cb = (float *)malloc(sizeof(float) * height), *co = (float *)malloc(sizeof(float) * height);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long x = 0; x < (long)width; x++) {
            for (size_t y = 0; y < height; y++) cb[y] = in[y * width + x];
            idct_1d_ws(&wc, cb, co);
            for (size_t y = 0; y < height; y++) temp[y * width + x] = co[y];
        }
        free(cb); free(co); ws_free(&wc);
#ifdef _OPENMP
#pragma omp barrier
#endif
        dct_ws wr; ws_init(&wr, width);
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long y = 0; y < (long)height; y++) idct_1d_ws(&wr, temp + y * width, out + y * width);
        ws_free(&wr);
    }
    free(temp);
}

/* ======================================================================
 * Spectral top-k selection + bitmap (compressive.rs:140-172)
 * ====================================================================== */

/* compressive.rs:152: ((n as f32 * ratio) as usize).max(1) */
size_t orc_retain_count(size_t n, float ratio) {
    float p = (float)n * ratio;
    size_t k = p <= 0.0f ? 0 : (size_t)p;
    return k < 1 ? 1 : k;
}

static inline uint32_t absbits(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return b & 0x7fffffffu;
}

/*
 * The reference stable-sorts (index, |c|) by |c| descending and keeps the
 * first k, i.e. the k largest magnitudes with ties going to the lower index.
 * Same set by radix select on the magnitude bits + an index-ordered tie scan.
 * Writes the LSB-first bitmap (bit idx%8 of byte idx/8, compressive.rs:157-163)
 * and returns the number of set bits (== k).  NaN coefficients are outside
 * the reference's defined ordering and are not supported.
 */
size_t orc_topk_bitmap(const float *c, size_t n, size_t k, uint8_t *bitmap, int threads) {
    memset(bitmap, 0, (n + 7) / 8);
    if (k == 0 || n == 0) return 0;
    if (k > n) k = n;
    uint64_t *hist = (uint64_t *)calloc(65536, sizeof(uint64_t));
    /* pass 1: top 16 bits */
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
    {
        uint64_t *h = (uint64_t *)calloc(65536, sizeof(uint64_t));
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long i = 0; i < (long)n; i++) h[absbits(c[i]) >> 16]++;
#ifdef _OPENMP
#pragma omp critical
#endif
        for (int j = 0; j < 65536; j++) hist[j] += h[j];
        free(h);
    }
    size_t above = 0; /* count strictly above the selected bucket */
    int hb = 65535;
    for (; hb >= 0; hb--) {
        if (above + hist[hb] >= k) break;
        above += hist[hb];
    }
    /* pass 2: low 16 bits inside bucket hb */
    memset(hist, 0, 65536 * sizeof(uint64_t));
    for (size_t i = 0; i < n; i++) {
        uint32_t b = absbits(c[i]);
        if ((int)(b >> 16) == hb) hist[b & 0xffff]++;
    }
    int lb = 65535;
    for (; lb >= 0; lb--) {
        if (above + hist[lb] >= k) break;
        above += hist[lb];
    }
    free(hist);
    uint32_t thr = ((uint32_t)hb << 16) | (uint32_t)lb;
    size_t need_eq = k - above, taken = 0, cnt = 0;
    for (size_t i = 0; i < n; i++) {
        uint32_t b = absbits(c[i]);
        int keep = b > thr || (b == thr && taken < need_eq);
        if (b == thr && keep) taken++;
        if (keep) { bitmap[i >> 3] |= (uint8_t)(1u << (i & 7)); cnt++; }
    }
    return cnt;
}

/* Retained values in ascending index order (compressive.rs:167-172). */
size_t orc_gather_retained(const float *c, size_t n, const uint8_t *bitmap, float *vals) {
    size_t j = 0;
    for (size_t i = 0; i < n; i++)
        if (bitmap[i >> 3] & (1u << (i & 7))) vals[j++] = c[i];
    return j;
}

/* Bitmap-rank scatter: dense[i] = vals[rank(i)] where bit i is set, else 0
 * (CompressiveSpectralDecoder::reconstruct, compressive.rs:732-752;
 * ref/c/hct_decoder.h:357-380). */
size_t orc_scatter_retained(const float *vals, size_t nvals, const uint8_t *bitmap, size_t n, float *dense) {
    size_t j = 0;
    for (size_t i = 0; i < n; i++) {
        if ((bitmap[i >> 3] & (1u << (i & 7))) && j < nvals) dense[i] = vals[j++];
        else dense[i] = 0.0f;
    }
    return j;
}

size_t orc_popcount_bytes(const uint8_t *p, size_t nbytes) {
    size_t c = 0;
    for (size_t i = 0; i < nbytes; i++) c += (size_t)__builtin_popcount(p[i]);
    return c;
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
