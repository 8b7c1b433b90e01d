// Writer side of the HCT path (host code): the LZ4 block compressor that
// produces the blocks the GPU decoder consumes.
//
// Restates crates/haagenti-lz4/src/block.rs:73-256 (compress_block): greedy
// LZ4 with a 64 Ki-entry multiplicative hash (u32 * 2654435761 >> 16), no
// match at position 0, 65535-byte window, 5 trailing literals, and the
// input_pos-2 hash refresh after each match.  Blocks are chunked as
// HctWriter::compress_data does (crates/haagenti-hct/src/tensor.rs:556-562).
// The reference clears its hash table per call; a generation tag per entry
// gives identical lookups without re-zeroing 512 KiB per 16 KiB block.
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include "../../include/hct_b200.h"

namespace {

constexpr size_t MIN_MATCH = 4, HASH_SIZE = 1u << 16, LAST_LITERALS = 5, MIN_INPUT = 13;

inline uint32_t rd32(const uint8_t *p) {
    uint32_t v;
    memcpy(&v, p, 4);
    return v;  // little-endian host
}
inline size_t hash4(uint32_t v) { return (size_t)((v * 2654435761u) >> 16) & (HASH_SIZE - 1); }

struct Table {
    std::vector<uint32_t> pos, gen;
    uint32_t cur = 0;
    Table() : pos(HASH_SIZE, 0), gen(HASH_SIZE, 0) {}
    void next() {
        if (++cur == 0) {
            std::fill(gen.begin(), gen.end(), 0);
            cur = 1;
        }
    }
    size_t get(size_t h) const { return gen[h] == cur ? pos[h] : 0; }
    void put(size_t h, size_t p) {
        pos[h] = (uint32_t)p;
        gen[h] = cur;
    }
};

bool put_len(uint8_t *out, size_t cap, size_t &o, size_t rem) {
    while (rem >= 255) {
        if (o >= cap) return false;
        out[o++] = 255;
        rem -= 255;
    }
    if (o >= cap) return false;
    out[o++] = (uint8_t)rem;
    return true;
}

// Returns HCT_B200_OK or HCT_B200_ERR_BUFFER_TOO_SMALL (write_sequence's check).
int compress(const uint8_t *in, size_t n, uint8_t *out, size_t cap, size_t *out_len, Table &t) {
    size_t o = 0;
    auto last_literals = [&](size_t anchor, size_t lit) -> int {
        size_t needed = 1 + lit / 255 + 1 + lit;
        if (o + needed > cap) return HCT_B200_ERR_BUFFER_TOO_SMALL;
        out[o++] = (uint8_t)((lit < 15 ? lit : 15) << 4);
        if (lit >= 15 && !put_len(out, cap, o, lit - 15)) return HCT_B200_ERR_BUFFER_TOO_SMALL;
        memcpy(out + o, in + anchor, lit);
        o += lit;
        return HCT_B200_OK;
    };
    if (n < MIN_INPUT) {
        int rc = last_literals(0, n);
        *out_len = o;
        return rc;
    }
    t.next();
    size_t ip = 0, anchor = 0;
    const size_t match_limit = n > LAST_LITERALS ? n - LAST_LITERALS : 0;
    const size_t mf_limit = match_limit > MIN_MATCH ? match_limit - MIN_MATCH : 0;
    while (ip < mf_limit) {
        const uint32_t cur = rd32(in + ip);
        const size_t h = hash4(cur);
        const size_t mp = t.get(h);
        t.put(h, ip);
        if (mp > 0 && ip - mp <= 65535 && rd32(in + mp) == cur) {
            size_t p1 = mp + MIN_MATCH, p2 = ip + MIN_MATCH;
            while (p2 < match_limit && in[p1] == in[p2]) { p1++; p2++; }
            const size_t ml = p2 - ip;
            const size_t lit = ip - anchor;
            const size_t needed = 1 + lit / 255 + 1 + lit + 2 + (ml - MIN_MATCH) / 255 + 1;
            if (o + needed > cap) {
                *out_len = o;
                return HCT_B200_ERR_BUFFER_TOO_SMALL;
            }
            const size_t lt = lit < 15 ? lit : 15, mt = (ml - MIN_MATCH) < 15 ? ml - MIN_MATCH : 15;
            out[o++] = (uint8_t)((lt << 4) | mt);
            if (lit >= 15) put_len(out, cap, o, lit - 15);
            memcpy(out + o, in + anchor, lit);
            o += lit;
            const uint16_t off = (uint16_t)(ip - mp);
            out[o++] = (uint8_t)(off & 0xff);
            out[o++] = (uint8_t)(off >> 8);
            if (ml - MIN_MATCH >= 15) put_len(out, cap, o, ml - MIN_MATCH - 15);
            ip += ml;
            anchor = ip;
            if (ip < mf_limit) t.put(hash4(rd32(in + ip - 2)), ip - 2);
        } else {
            ip += 1;
        }
    }
    int rc = HCT_B200_OK;
    if (n > anchor) rc = last_literals(anchor, n - anchor);
    *out_len = o;
    return rc;
}


// quantization.rs:136-163: truncating, flush-to-zero f32 -> f16 bits.
uint16_t f32_to_f16_trunc(float val) {
    uint32_t bits;
    memcpy(&bits, &val, 4);
    const uint32_t sign = (bits >> 31) & 1, frac = bits & 0x7fffff;
    const int32_t exp = (int32_t)((bits >> 23) & 0xff);
    if (exp == 0) return (uint16_t)(sign << 15);
    if (exp == 0xff) return (uint16_t)((sign << 15) | (0x1f << 10) | (frac >> 13));
    const int32_t ne = exp - 127 + 15;
    if (ne >= 31) return (uint16_t)((sign << 15) | (0x1f << 10));
    if (ne <= 0) return (uint16_t)(sign << 15);
    return (uint16_t)((sign << 15) | ((uint32_t)ne << 10) | (frac >> 13));
}

// Rust `(x).round() as i8`: half away from zero, saturating, NaN -> 0.
inline int round_i8(float x) {
    const float r = std::round(x);
    if (r != r) return 0;
    if (r < -128.0f) return -128;
    if (r > 127.0f) return 127;
    return (int)r;
}

inline uint32_t mag_bits(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return b & 0x7fffffffu;
}

}  // namespace

namespace {

// quantization.rs:30-70 (one OpenMP task per 32-element block), the scale
// stored through ScaleBits.
template <uint16_t (*ScaleBits)(float)>
int quantize_int4_impl(const float *w, size_t n, uint8_t *out) {
    if (n == 0) return HCT_B200_OK;
    if (!w || !out) return HCT_B200_ERR_INVALID_ARGUMENT;
    const size_t nb = (n + 31) / 32;
    uint8_t *nib = out + 2 * nb;
#pragma omp parallel for schedule(static)
    for (long b = 0; b < (long)nb; b++) {
        const size_t s = (size_t)b * 32, e = s + 32 < n ? s + 32 : n;
        float max_abs = 0.0f;
        for (size_t i = s; i < e; i++) max_abs = std::fmax(max_abs, std::fabs(w[i]));
        const float scale = max_abs > 1e-10f ? max_abs / 7.0f : 1.0f;
        const uint16_t h = ScaleBits(scale);
        out[2 * b] = (uint8_t)(h & 0xff);
        out[2 * b + 1] = (uint8_t)(h >> 8);
        // a 32-element block spans 16 whole nibble bytes, so threads never share a byte
        for (size_t i = s; i < e; i++) {
            int q = round_i8(w[i] / scale);
            q = q < -8 ? -8 : (q > 7 ? 7 : q);
            const uint8_t v = (uint8_t)(q + 8);
            if (i & 1) nib[i >> 1] |= (uint8_t)((v & 0x0f) << 4);
            else nib[i >> 1] = (uint8_t)(v & 0x0f);
        }
    }
    return HCT_B200_OK;
}

// half::f16::from_f32 (round-to-nearest-even), as mixed_precision.rs:463
uint16_t f32_to_f16_rne(float v) { return __half_as_ushort(__float2half_rn(v)); }

}  // namespace

extern "C" {

// quantization.rs:30-70: truncating, flush-to-zero f16 scales.
int hct_b200_quantize_int4(const float *w, size_t n, uint8_t *out) {
    return quantize_int4_impl<f32_to_f16_trunc>(w, n, out);
}

// mixed_precision.rs:448-486: the same blocks with round-to-nearest-even scales.
int hct_b200_quantize_int4_mp(const float *w, size_t n, uint8_t *out) {
    return quantize_int4_impl<f32_to_f16_rne>(w, n, out);
}

// compressive.rs:140-172: keep the k largest |c| (ties to the lower index),
// LSB-first bitmap, retained values in ascending index order.  `bitmap`
// holds ceil(n/8) bytes, `values` k floats.
int hct_b200_spectral_select(const float *c, size_t n, size_t k, uint8_t *bitmap, float *values,
                             size_t *count) {
    if (!count || (n && (!c || !bitmap || !values))) return HCT_B200_ERR_INVALID_ARGUMENT;
    *count = 0;
    const size_t nbytes = (n + 7) / 8;
    memset(bitmap, 0, nbytes);
    if (n == 0 || k == 0) return HCT_B200_OK;
    if (k > n) k = n;
    // radix select of the k-th largest magnitude: 16 high bits, then 16 low bits
    std::vector<uint64_t> hist(65536, 0);
#pragma omp parallel
    {
        std::vector<uint64_t> h(65536, 0);
#pragma omp for schedule(static) nowait
        for (long i = 0; i < (long)n; i++) h[mag_bits(c[i]) >> 16]++;
#pragma omp critical
        for (int j = 0; j < 65536; j++) hist[j] += h[j];
    }
    uint64_t above = 0;
    int hb = 65535;
    for (; hb > 0 && above + hist[hb] < k; hb--) above += hist[hb];
    std::fill(hist.begin(), hist.end(), 0);
#pragma omp parallel
    {
        std::vector<uint64_t> h(65536, 0);
#pragma omp for schedule(static) nowait
        for (long i = 0; i < (long)n; i++) {
            const uint32_t b = mag_bits(c[i]);
            if ((int)(b >> 16) == hb) h[b & 0xffff]++;
        }
#pragma omp critical
        for (int j = 0; j < 65536; j++) hist[j] += h[j];
    }
    int lb = 65535;
    for (; lb > 0 && above + hist[lb] < k; lb--) above += hist[lb];
    const uint32_t thr = ((uint32_t)hb << 16) | (uint32_t)lb;
    const uint64_t need_eq = k - above;
    // index-ordered pass over 8-element bytes, parallel by byte ranges: the
    // ties taken are the first need_eq equal values in index order
    const long nchunk = 256;
    std::vector<uint64_t> eq_before(nchunk + 1, 0), kept_before(nchunk + 1, 0);
    const size_t per = (nbytes + nchunk - 1) / nchunk;
#pragma omp parallel for schedule(static)
    for (long t = 0; t < nchunk; t++) {
        const size_t i0 = std::min(n, (size_t)t * per * 8), i1 = std::min(n, (size_t)(t + 1) * per * 8);
        uint64_t e = 0;
        for (size_t i = i0; i < i1; i++) e += mag_bits(c[i]) == thr;
        eq_before[t + 1] = e;
    }
    for (long t = 0; t < nchunk; t++) eq_before[t + 1] += eq_before[t];
#pragma omp parallel for schedule(static)
    for (long t = 0; t < nchunk; t++) {
        const size_t i0 = std::min(n, (size_t)t * per * 8), i1 = std::min(n, (size_t)(t + 1) * per * 8);
        uint64_t eq = eq_before[t], kept = 0;
        for (size_t i = i0; i < i1; i++) {
            const uint32_t b = mag_bits(c[i]);
            bool keep = b > thr;
            if (b == thr) keep = eq++ < need_eq;
            if (keep) {
                bitmap[i >> 3] |= (uint8_t)(1u << (i & 7));
                kept++;
            }
        }
        kept_before[t + 1] = kept;
    }
    for (long t = 0; t < nchunk; t++) kept_before[t + 1] += kept_before[t];
#pragma omp parallel for schedule(static)
    for (long t = 0; t < nchunk; t++) {
        const size_t i0 = std::min(n, (size_t)t * per * 8), i1 = std::min(n, (size_t)(t + 1) * per * 8);
        uint64_t j = kept_before[t];
        for (size_t i = i0; i < i1; i++)
            if (bitmap[i >> 3] >> (i & 7) & 1) values[j++] = c[i];
    }
    *count = kept_before[nchunk];
    return HCT_B200_OK;
}

size_t hct_b200_lz4_max_compressed_size(size_t n) { return n + n / 255 + 16; }

int hct_b200_lz4_compress_block(const uint8_t *in, size_t in_len, uint8_t *out, size_t out_cap,
                                size_t *out_len) {
    if ((!in && in_len) || !out || !out_len) return HCT_B200_ERR_INVALID_ARGUMENT;
    static thread_local Table t;
    return compress(in, in_len, out, out_cap, out_len, t);
}

int hct_b200_lz4_compress_chunks(const uint8_t *in, size_t in_len, size_t block_size,
                                 uint8_t *out, size_t out_stride, uint32_t *lens) {
    if ((!in && in_len) || !out || !lens || block_size == 0) return HCT_B200_ERR_INVALID_ARGUMENT;
    const size_t nb = in_len == 0 ? 0 : (in_len + block_size - 1) / block_size;
    int bad = 0;
#pragma omp parallel for schedule(dynamic, 8) reduction(| : bad)
    for (long i = 0; i < (long)nb; i++) {
        static thread_local Table t;
        const size_t s = (size_t)i * block_size;
        const size_t len = in_len - s < block_size ? in_len - s : block_size;
        size_t ol = 0;
        bad |= compress(in + s, len, out + (size_t)i * out_stride, out_stride, &ol, t);
        lens[i] = (uint32_t)ol;
    }
    return bad;
}

}  // extern "C"
