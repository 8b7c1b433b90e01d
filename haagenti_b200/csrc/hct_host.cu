// Host side of libhct_b200.so: the C ABI declared in include/hct_b200.h.
//
// This is the C++ counterpart of the reference's Rust host code for the
// decode path: the Decompressor trait surface of Lz4Decompressor
// (crates/haagenti-lz4/src/decompress.rs:28-73), dequantize_int4
// (crates/haagenti/src/testing/quantization.rs:82-131), and the HCT readers
// (crates/haagenti-hct/src/tensor.rs:408-516, 832-1021).  Container parsing
// stays on the host; every byte of payload work runs in the CUDA kernels of
// lz4_decode.cu, int4_dequant.cu and idct_gemm.cu.  There is no CPU decode
// path: without a device the calls fail with HCT_B200_ERR_NO_DEVICE.
#include <dlfcn.h>

#include <cstdarg>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "common.cuh"

using namespace hct;

namespace {

// ---- small utilities -------------------------------------------------------

struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
    DevBuf() = default;
    DevBuf(const DevBuf &) = delete;
    DevBuf &operator=(const DevBuf &) = delete;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    // Grows (never shrinks); contents are not preserved.
    cudaError_t reserve(size_t bytes) {
        if (bytes <= cap && p) return cudaSuccess;
        release();
        size_t want = bytes < 256 ? 256 : bytes;
        cudaError_t e = cudaMalloc(&p, want);
        if (e != cudaSuccess) {
            p = nullptr;
            return e;
        }
        cap = want;
        return cudaSuccess;
    }
    template <class T>
    T *as() const {
        return reinterpret_cast<T *>(p);
    }
};

inline uint64_t round_up(uint64_t v, uint64_t m) { return (v + m - 1) / m * m; }

void set_err(hct_b200_error *err, int code, int block, uint64_t pos, uint64_t req, uint64_t prov,
             const char *fmt, ...) __attribute__((format(printf, 7, 8)));

void set_err(hct_b200_error *err, int code, int block, uint64_t pos, uint64_t req, uint64_t prov,
             const char *fmt, ...) {
    if (!err) return;
    err->code = code;
    err->block = block;
    err->position = pos;
    err->required = req;
    err->provided = prov;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(err->message, sizeof(err->message), fmt, ap);
    va_end(ap);
}

void clear_err(hct_b200_error *err) {
    if (!err) return;
    memset(err, 0, sizeof(*err));
    err->block = -1;
}

int cuda_code(cudaError_t e) {
    if (e == cudaSuccess) return HCT_B200_OK;
    if (e == cudaErrorMemoryAllocation) return HCT_B200_ERR_OUT_OF_MEMORY;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return HCT_B200_ERR_NO_DEVICE;
    return HCT_B200_ERR_CUDA;
}

#define CK(expr)                                                                       \
    do {                                                                               \
        cudaError_t _e = (expr);                                                       \
        if (_e != cudaSuccess) {                                                       \
            set_err(err, cuda_code(_e), -1, 0, 0, 0, "%s: %s", #expr, cudaGetErrorString(_e)); \
            return cuda_code(_e);                                                      \
        }                                                                              \
    } while (0)

// XXH3-64 comes from the system libxxhash (the reference uses xxhash-rust
// 0.8.15, same algorithm); resolved at run time so the library loads
// without it and only checksum validation needs it.
using Xxh3Fn = unsigned long long (*)(const void *, size_t);
Xxh3Fn xxh3_fn() {
    static Xxh3Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *names[] = {"libxxhash.so.0", "libxxhash.so"};
        for (const char *n : names) {
            void *h = dlopen(n, RTLD_NOW | RTLD_LOCAL);
            if (h) {
                fn = reinterpret_cast<Xxh3Fn>(dlsym(h, "XXH3_64bits"));
                if (fn) break;
            }
        }
    });
    return fn;
}

inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
inline uint32_t rd32(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
inline uint64_t rd64(const uint8_t *p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

constexpr uint16_t FLAG_HEADER_CHECKSUM = 0x0001;  // tensor.rs:53
constexpr uint16_t FLAG_BLOCK_CHECKSUMS = 0x0002;  // tensor.rs:56
constexpr uint16_t FLAG_QUANTIZATION = 0x0004;     // tensor.rs:59

struct Basis {
    DevBuf buf;
    uint64_t ld = 0;
};

}  // namespace

// ---- context ---------------------------------------------------------------

// Per-launch timing records (CUDA events on the launching stream), kept only
// while profiling is enabled on the context.
enum ProfKind {
    PK_LZ4 = 0,
    PK_SCATTER = 1,
    PK_GEMM = 2,
    PK_DEQUANT = 3,
    PK_PACK = 4,
    PK_DFT1 = 5,
    PK_RANK = 6,
    PK_SPACK = 7,
    PK_DFT2 = 8,
    PK_COUNT = 9
};
static const char *const kProfNames[PK_COUNT] = {
    "lz4_decode_blocks", "spectral_scatter", "umma_gemm",     "dequant_int4", "makhoul_pack",
    "dft_stage1",        "spectral_rank",    "spectral_pack", "dft_stage2"};
struct ProfRec {
    int kind;
    cudaEvent_t a, b;
    double work;  // algorithmic flops (umma_gemm) or bytes (the others)
};

struct hct_b200_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;  // used by the host-buffer entry points
    // front-end stream of the readers' asynchronous decodes (LZ4 + bitmap
    // rank), so that a tensor's front end overlaps the IDCT of the previous one
    cudaStream_t side = nullptr;
    DevBuf dense, tt, chunk, meta, flag;
    DevBuf za, zb;  // factored-IDCT intermediates (rows*cols fp16 each)
    DevBuf sched;   // tile counters of the DFT stage kernels
    DevBuf zscratch, zsrc, zdst, zjob, zstatus;  // Zstandard decode
    DevBuf io_in, io_out, io_blk, io_status;
    std::map<uint64_t, std::unique_ptr<Basis>> bases;
    std::map<uint64_t, std::unique_ptr<DevBuf>> dft_mats;  // realified n-point DFT (n, ld), fp16
    std::map<uint32_t, std::unique_ptr<DevBuf>> twiddles;  // e^{2 pi i j / H}, complex f32
    std::map<uint32_t, std::unique_ptr<DevBuf>> pack_tabs;  // Makhoul-pack twiddles per length
    std::map<uint64_t, std::unique_ptr<DevBuf>> fold_tabs;  // per-k2 stage-1 matrices (P, Q, rows)
    std::map<uint64_t, std::unique_ptr<DevBuf>> mfold_tabs;  // mode-6 per-pair matrices (P, Q)
    DevBuf cos_tbl;
    int idct_mode = HCT_B200_IDCT_AUTO;
    bool profiling = false;
    std::vector<ProfRec> prof;
    std::vector<cudaEvent_t> event_pool;
    size_t pool_used = 0;

    cudaEvent_t event() {
        if (pool_used == event_pool.size()) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
            event_pool.push_back(e);
        }
        return event_pool[pool_used++];
    }
    // Brackets one launch: call begin() before and end() after it.
    int prof_begin(cudaStream_t s) {
        if (!profiling) return -1;
        ProfRec r{0, event(), event(), 0.0};
        if (!r.a || !r.b) return -1;
        cudaEventRecord(r.a, s);
        prof.push_back(r);
        return (int)prof.size() - 1;
    }
    void prof_end(int slot, int kind, double work, cudaStream_t s) {
        if (slot < 0) return;
        prof[slot].kind = kind;
        prof[slot].work = work;
        cudaEventRecord(prof[slot].b, s);
    }
};

// A parsed V3 fragment container on the device: each fragment's bitmap and
// fp16 values copied to 16-byte aligned places of d_data.
struct hct_b200_v3 {
    struct Frag {
        size_t bm_off, vals_off;
        uint64_t nvals;
    };
    hct_b200_ctx *ctx = nullptr;
    uint64_t rows = 0, cols = 0;  // of the transform (a column vector is one row)
    DevBuf d_data;
    std::vector<Frag> frags;
};

// A parsed HoloTensor file: the header, one record per fragment index entry
// (what read_fragment + add_fragment would make of it), and the f32 values
// of its SV03 fragments on the device.
struct hct_b200_holo {
    enum Kind {
        SV03 = 0,
        PAST_END,    // the stored bytes run past the file ("failed to read fragment data")
        ZSTD_BAD,    // entry flag bit 0 and the zstd frames did not decode
        SHORT,       // fewer than 8 bytes ("fragment too short")
        V3_SHORT,    // SV03 magic, fewer than 20 bytes ("V3 fragment too short")
        LEGACY,      // the V1 or V2 spectral layouts
    };
    struct Frag {
        uint16_t index = 0;
        Kind kind = SV03;
        bool checksum_ok = true;
        uint32_t num_coeffs = 0, F = 0, start = 0;
        uint64_t count = 0;  // values add_fragment_v3 writes (before its position < n check)
        uint64_t dev_off = 0;  // f32 elements into d_vals
    };
    hct_b200_ctx *ctx = nullptr;
    hct_b200_holo_info hdr{};
    std::vector<Frag> frags;  // index-table order; the inline form has one
    uint64_t rows = 0, cols = 0;  // of the transform (a column vector is one row)
    DevBuf d_vals, d_res;
};

struct hct_b200_reader {
    hct_b200_ctx *ctx = nullptr;
    hct_b200_header hdr{};
    std::vector<uint32_t> offsets, sizes;
    std::vector<uint64_t> checksums;
    size_t data_offset = 0;  // within the file
    size_t data_len = 0;
    uint64_t max_block = 0;  // largest compressed block
    DevBuf d_data, d_blocks, d_status;
    std::vector<uint32_t> expected;
    uint64_t rows = 0, cols = 0;
    bool spectral = false;
    // deferred status of an asynchronous decode (pinned host copies)
    hct_b200_status *h_status = nullptr;
    int *h_flag = nullptr;
    cudaEvent_t done = nullptr;
    bool pending = false;
    uint64_t pending_elems = 0;  // INT4 elements a plain decode produced (0 = spectral)
    // Cross-stream ordering of d_data: an upload on any stream waits for the
    // last LZ4 launch that read the buffer (data_free), and an LZ4 launch
    // waits for the last upload (uploaded).  Uploads on a copy stream thus
    // overlap the decode of other tensors without host synchronisation.
    cudaEvent_t uploaded = nullptr, data_free = nullptr;
    bool upload_pending = false, read_pending = false;
    // the reader's own decoded payload, rank directory and error flag: the
    // front end of decode_async fills them on ctx->side (front_done), the back
    // end consumes them on the caller's stream (back_done)
    DevBuf d_payload, d_chunk, d_meta, d_flag;
    cudaEvent_t front_done = nullptr, back_done = nullptr;
    bool back_pending = false;
    ~hct_b200_reader() {
        if (h_status) cudaFreeHost(h_status);
        if (h_flag) cudaFreeHost(h_flag);
        if (done) cudaEventDestroy(done);
        if (uploaded) cudaEventDestroy(uploaded);
        if (data_free) cudaEventDestroy(data_free);
        if (front_done) cudaEventDestroy(front_done);
        if (back_done) cudaEventDestroy(back_done);
    }
    // stream s is about to read d_data (LZ4)
    cudaError_t before_read(cudaStream_t s) {
        return upload_pending ? cudaStreamWaitEvent(s, uploaded, 0) : cudaSuccess;
    }
    // stream s has enqueued its last read of d_data
    cudaError_t after_read(cudaStream_t s) {
        read_pending = true;
        return cudaEventRecord(data_free, s);
    }
};

namespace {

// Stage 1 with the twiddle folded into per-k2 matrices where the shapes allow.
#ifndef FDCT_FOLD_TWIDDLE
#define FDCT_FOLD_TWIDDLE 1
#endif
// The second pass's Makhoul pack folded into its stage 1 (stage mode 6) where
// the shapes allow.
#ifndef FDCT_FOLD_MAKHOUL
#define FDCT_FOLD_MAKHOUL 1
#endif
// ... and the first pass's, from a spectral payload
#ifndef FDCT_FOLD_ROW
#define FDCT_FOLD_ROW 1
#endif

int ensure_device(hct_b200_ctx *ctx) {
    cudaError_t e = cudaSetDevice(ctx->device);
    return cuda_code(e);
}

// Cached fp16 DCT-III basis of length n (row stride round_up(n, 8)).
int get_basis(hct_b200_ctx *ctx, uint64_t n, const Basis **out, cudaStream_t s,
              hct_b200_error *err) {
    auto it = ctx->bases.find(n);
    if (it != ctx->bases.end()) {
        *out = it->second.get();
        return HCT_B200_OK;
    }
    auto b = std::make_unique<Basis>();
    b->ld = round_up(n, 8);
    CK(b->buf.reserve(n * b->ld * 2));
    // cos(pi j / 2n), j < 4n, in f64 from libm on the host
    std::vector<double> tbl(4 * n);
    for (uint64_t j = 0; j < 4 * n; j++) tbl[j] = std::cos(M_PI * (double)j / (2.0 * (double)n));
    CK(ctx->cos_tbl.reserve(tbl.size() * sizeof(double)));
    CK(cudaMemcpyAsync(ctx->cos_tbl.p, tbl.data(), tbl.size() * sizeof(double),
                       cudaMemcpyHostToDevice, s));
    CK(launch_basis(ctx->cos_tbl.as<double>(), n, b->buf.as<half_bits>(), b->ld, s));
    CK(cudaStreamSynchronize(s));  // tbl is released on return
    *out = b.get();
    ctx->bases[n] = std::move(b);
    return HCT_B200_OK;
}

// Bytes of the pack output Z for `batch` rows of length L (rows of
// fdct_padded_p(P) complex fp16 per (b, k2)); 0 when L does not factor.
uint64_t fdct_z_bytes(uint64_t batch, uint64_t L) {
    uint32_t P = 0, Q = 0;
    if (!fdct_factor(L, &P, &Q)) return 0;
    return batch * Q * (uint64_t)fdct_padded_p(P) * 4;
}

int reserve_spectral(hct_b200_ctx *ctx, uint64_t rows, uint64_t cols,
                     hct_b200_error *err) {
    CK(ctx->dense.reserve(rows * round_up(cols, 8) * 2 + 16));
    CK(ctx->tt.reserve(cols * round_up(rows, 8) * 2 + 16));
    CK(ctx->za.reserve(std::max<uint64_t>(
        rows * cols * 2, std::max(fdct_z_bytes(rows, cols), fdct_z_bytes(cols, rows))) + 16));
    CK(ctx->zb.reserve(rows * cols * 2 + 16));
    CK(ctx->chunk.reserve(rank_dir_words(rows * cols) * sizeof(uint32_t)));
    CK(ctx->meta.reserve(4 * sizeof(uint64_t)));
    CK(ctx->flag.reserve(sizeof(int)));
    return HCT_B200_OK;
}

// The two contractions on a dense fp16 coefficient matrix held in ctx->dense
// (rows x round_up(cols, 8)).
// Realified n-point DFT matrix, 2n rows of ld >= 2n fp16 (zero columns past 2n).
int get_dft_matrix(hct_b200_ctx *ctx, uint32_t n, uint32_t ld, const half_bits **out,
                   cudaStream_t s, hct_b200_error *err) {
    const uint64_t key = (uint64_t)n | ((uint64_t)ld << 32);
    auto it = ctx->dft_mats.find(key);
    if (it == ctx->dft_mats.end()) {
        auto b = std::make_unique<DevBuf>();
        CK(b->reserve((size_t)2 * n * ld * 2));
        CK(launch_dft_matrix(n, 2 * n, ld, b->as<half_bits>(), s));
        it = ctx->dft_mats.emplace(key, std::move(b)).first;
    }
    *out = it->second->as<half_bits>();
    return HCT_B200_OK;
}


int get_twiddle(hct_b200_ctx *ctx, uint32_t H, const float **out, cudaStream_t s,
                hct_b200_error *err) {
    auto it = ctx->twiddles.find(H);
    if (it == ctx->twiddles.end()) {
        auto b = std::make_unique<DevBuf>();
        CK(b->reserve((size_t)H * 8));
        CK(launch_twiddle_table(H, b->as<float>(), s));
        it = ctx->twiddles.emplace(H, std::move(b)).first;
    }
    *out = it->second->as<float>();
    return HCT_B200_OK;
}

// Where a decode keeps the rank directory of its spectral payload and its
// device error flag: the context's scratch for the one-shot entry points, a
// reader's own buffers for its asynchronous decode (ranked = the directory
// was already built by the reader's front end).
struct RankDir {
    uint32_t *chunk;
    uint64_t *meta;
    int *flag;
    bool ranked;
};

RankDir ctx_rank_dir(hct_b200_ctx *ctx) {
    return RankDir{ctx->chunk.as<uint32_t>(), ctx->meta.as<uint64_t>(), ctx->flag.as<int>(), false};
}

// Whether run_idct takes the factored path for a rows x cols matrix, and
// whether it then decodes a spectral payload straight into the row pack.
bool idct_factored(const hct_b200_ctx *ctx, uint64_t rows, uint64_t cols, uint32_t *pn,
                   uint32_t *qn, uint32_t *pm, uint32_t *qm) {
    return ctx->idct_mode != HCT_B200_IDCT_DENSE && fdct_factor(cols, pn, qn) &&
           (rows == 1 || fdct_factor(rows, pm, qm));
}
bool spectral_fused(const hct_b200_ctx *ctx, uint64_t rows, uint64_t cols) {
    uint32_t a, b, c, d;
    return ctx->idct_mode == HCT_B200_IDCT_AUTO && idct_factored(ctx, rows, cols, &a, &b, &c, &d) &&
           spectral_pack_supported(cols);
}

// Whether a pass over `batch` lines of length 2 P Q can take the Makhoul
// pack folded into stage 1 (stage mode 6 reading the previous pass's
// transposed output in the permuted line order, then stage 2 as mode 5).
bool makhoul_fold_ok(uint64_t batch, uint32_t P, uint32_t Q) {
    return FDCT_FOLD_MAKHOUL && FDCT_FOLD_TWIDDLE && batch % 128 == 0 && P % 4 == 0 &&
           2 * P >= 64 && 2 * P <= 128 && Q % 32 == 0 && 2 * Q <= 256;
}

// Options of one pass: the slot order its pack writes the lines in (for a
// next pass with the Makhoul fold; perm_q = 0 keeps line b at slot b), and
// whether this pass is such a next pass (its input `in` then holds the lines
// as T'[n][k2][r] and no pack runs).
struct AxisOpts {
    uint32_t perm_q = 0, perm_2p = 0;
    bool makhoul_fold = false;
};

// One axis of the factored IDCT: rows of length L (fp16, stride ld_in) in
// `in`, batch rows; the result is written transposed, out[n * ldo + slot(b)], in
// out_dtype (pack -> DFT stage 1 -> DFT stage 2, see fdct.cu).
// The pack reads dense fp16 rows (`in`, stride ld_in) or, when `payload` is
// set, decodes the rows straight from a spectral payload whose rank directory
// launch_spectral_rank has put in dir.chunk / dir.meta.
int fdct_axis(hct_b200_ctx *ctx, const half_bits *in, uint64_t ld_in, const uint8_t *payload,
              const RankDir &dir, uint64_t batch, uint64_t L, uint32_t P, uint32_t Q, void *out,
              uint64_t ldo, int out_dtype, cudaStream_t s, hct_b200_error *err,
              const AxisOpts &opt = AxisOpts()) {
    const uint32_t H = (uint32_t)(L / 2);
    const uint32_t Pp = fdct_padded_p(P);  // Z rows: Pp complex, zeros past P
    const half_bits *wp = nullptr, *wq = nullptr;
    const float *tw = nullptr;
    int rc = get_dft_matrix(ctx, P, 2 * Pp, &wp, s, err);
    if (!rc) rc = get_dft_matrix(ctx, Q, 2 * Q, &wq, s, err);
    if (!rc) rc = get_twiddle(ctx, H, &tw, s, err);
    if (rc) return rc;
    auto pt = ctx->pack_tabs.find((uint32_t)L);
    if (pt == ctx->pack_tabs.end()) {
        auto b = std::make_unique<DevBuf>();
        CK(b->reserve((size_t)L * 12));
        CK(launch_pack_tables((uint32_t)L, P, Q, b->as<float>(), s));
        pt = ctx->pack_tabs.emplace((uint32_t)L, std::move(b)).first;
    }
    int *flag = dir.flag;
    const double elems = (double)batch * (double)L;
    CK(ctx->sched.reserve(64));
    GemmArgs g2{ctx->zb.as<half_bits>(), wq, (uint64_t)P * batch, 2ull * Q, 2ull * Q, batch,
                2ull * Q, out, ldo, 5, out_dtype, flag};
    g2.tile_counter = ctx->sched.as<uint32_t>() + 1;
    g2.P = P;
    g2.Q = Q;
    g2.H = H;
    g2.batch = batch;
    g2.scale = (float)std::sqrt(2.0 / (double)L);
    if (opt.makhoul_fold) {
        // no pack: stage 1 reads two columns of 128 lines of T' per tile and
        // multiplies them by the pair's matrix (Makhoul coefficients and
        // twiddle folded in), stage 2 as mode 5.  T' is the previous pass's
        // output (`in`), or, for a spectral payload, the decoded lines written
        // transposed by the spectral pack's TR variant.
        if (!makhoul_fold_ok(batch, P, Q)) {
            set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0,
                    "Makhoul fold: unsupported pass (P %u, Q %u, %llu lines)", P, Q,
                    (unsigned long long)batch);
            return HCT_B200_ERR_INVALID_ARGUMENT;
        }
        const uint32_t kbc = (2 * P + 63) / 64;
        const uint64_t key = ((uint64_t)P << 32) | Q;
        auto it = ctx->mfold_tabs.find(key);
        if (it == ctx->mfold_tabs.end()) {
            auto b = std::make_unique<DevBuf>();
            CK(b->reserve((size_t)(Q / 2 + 1) * 256 * 128 * kbc * 2));
            CK(launch_makhoul_fold_table(P, Q, kbc, b->as<half_bits>(), s));
            it = ctx->mfold_tabs.emplace(key, std::move(b)).first;
        }
        const half_bits *tin = in;
        uint64_t tld = ld_in;
        int slot = -1;
        if (payload) {
            const uint64_t bmb = (batch * L + 7) / 8;
            slot = ctx->prof_begin(s);
            CK(launch_spectral_pack(payload, bmb, dir.chunk, dir.meta, batch, (uint32_t)L, P, Q,
                                    pt->second->as<float>(), ctx->za.as<half_bits>(), false,
                                    opt.perm_q, opt.perm_2p, s, true));
            ctx->prof_end(slot, PK_SPACK, (double)bmb + 0.17 * elems + 2.0 * elems, s);
            tin = ctx->za.as<half_bits>();
            tld = L;
        }
        GemmArgs g1{tin, it->second->as<half_bits>(), (uint64_t)(Q / 2 + 1) * batch, 256,
                    128ull * kbc, tld, 128ull * kbc, ctx->zb.p, 0, 6, HCT_B200_F16, flag};
        g1.P = P;
        g1.Q = Q;
        g1.H = H;
        g1.batch = batch;
        slot = ctx->prof_begin(s);
        CK(launch_umma_gemm(g1, s));
        ctx->prof_end(slot, PK_DFT1, 4.0 * elems, s);
        slot = ctx->prof_begin(s);
        CK(launch_umma_gemm(g2, s));
        ctx->prof_end(slot, PK_DFT2, (2.0 + (out_dtype == HCT_B200_F32 ? 4.0 : 2.0)) * elems, s);
        return HCT_B200_OK;
    }
    // Twiddle folded into per-k2 stage-1 matrices (stage modes 4 and 5): Z is
    // written k2-major, stage 1 multiplies 128 lines of one k2 by that k2's
    // matrix and stores G[m1][k2][ri][b] without any epilogue arithmetic, and
    // stage 2 reads G as an MN-major operand.  Needs whole 128-line tiles per
    // k2 and K-row blocks of 64 (Q % 32 == 0) inside the stage kernel's sizes.
    const bool fold = FDCT_FOLD_TWIDDLE && batch % 128 == 0 && Q % 32 == 0 && 2 * Q <= 256 &&
                      2 * Pp <= 256;
    const half_bits *w4 = nullptr;
    if (fold) {
        const uint32_t wr = stage_w_rows(2ull * P, 2ull * Pp);
        const uint64_t key = ((uint64_t)P << 32) | ((uint64_t)Q << 16) | wr;
        auto it = ctx->fold_tabs.find(key);
        if (it == ctx->fold_tabs.end()) {
            auto b = std::make_unique<DevBuf>();
            CK(b->reserve((size_t)Q * wr * 2 * Pp * 2));
            CK(launch_twiddled_dft_table(P, Q, wr, 2 * Pp, b->as<half_bits>(), s));
            it = ctx->fold_tabs.emplace(key, std::move(b)).first;
        }
        w4 = it->second->as<half_bits>();
    }
    int slot = ctx->prof_begin(s);
    if (payload) {
        const uint64_t bmb = (batch * L + 7) / 8;
        CK(launch_spectral_pack(payload, bmb, dir.chunk, dir.meta,
                                batch, (uint32_t)L, P, Q, pt->second->as<float>(),
                                ctx->za.as<half_bits>(), fold, opt.perm_q, opt.perm_2p, s));
        // bitmap + ~0.3 of the INT4 section read, fp16 pairs written
        ctx->prof_end(slot, PK_SPACK, (double)bmb + 0.17 * elems + 2.0 * elems, s);
    } else {
        CK(launch_makhoul_pack(in, ld_in, batch, (uint32_t)L, P, Q, pt->second->as<float>(),
                               ctx->za.as<half_bits>(), fold, opt.perm_q, opt.perm_2p, s));
        ctx->prof_end(slot, PK_PACK, 4.0 * elems, s);
    }
    GemmArgs g1{ctx->za.as<half_bits>(), fold ? w4 : wp, batch * Q, 2ull * P, 2ull * Pp, 2ull * Pp,
                2ull * Pp, ctx->zb.p, 0, fold ? 4 : 2, HCT_B200_F16, flag};
    g1.tile_counter = ctx->sched.as<uint32_t>();
    g1.P = P;
    g1.Q = Q;
    g1.H = H;
    g1.batch = batch;
    g1.twiddle = tw;
    slot = ctx->prof_begin(s);
    CK(launch_umma_gemm(g1, s));
    ctx->prof_end(slot, PK_DFT1, 4.0 * elems, s);
    if (!fold) {
        g2.lda = 2ull * Q;
        g2.mode = 3;
    }
    slot = ctx->prof_begin(s);
    CK(launch_umma_gemm(g2, s));
    ctx->prof_end(slot, PK_DFT2, (2.0 + (out_dtype == HCT_B200_F32 ? 4.0 : 2.0)) * elems, s);
    return HCT_B200_OK;
}

// IDCT of a rows x cols coefficient matrix.  The coefficients are either the
// dense fp16 matrix in ctx->dense (payload == nullptr) or a spectral payload
// on the device, which is decoded into the first pass of the factored path
// when the row length allows, and scattered into ctx->dense otherwise.
int run_idct(hct_b200_ctx *ctx, uint64_t rows, uint64_t cols, void *d_out, int out_dtype,
             cudaStream_t s, hct_b200_error *err, const uint8_t *payload = nullptr,
             size_t payload_len = 0, const RankDir *dir_in = nullptr) {
    const uint64_t ldw = round_up(cols, 8), ldh = round_up(rows, 8);
    const RankDir dir = dir_in ? *dir_in : ctx_rank_dir(ctx);
    int *flag = dir.flag;
    uint32_t pn = 0, qn = 0, pm = 0, qm = 0;
    const bool factored = idct_factored(ctx, rows, cols, &pn, &qn, &pm, &qm);
    const uint8_t *src = nullptr;
    if (payload) {
        const uint64_t total = rows * cols;
        if (spectral_fused(ctx, rows, cols)) {
            if (!dir.ranked) {
                int slot = ctx->prof_begin(s);
                CK(launch_spectral_rank(payload, payload_len, total, dir.chunk, dir.meta, flag, s));
                ctx->prof_end(slot, PK_RANK, (double)((total + 7) / 8), s);
            }
            src = payload;
        } else {
            int slot = ctx->prof_begin(s);
            CK(launch_spectral_scatter(payload, payload_len, rows, cols, dir.chunk, dir.meta,
                                       ctx->dense.as<half_bits>(), ldw, flag, s));
            ctx->prof_end(slot, PK_SCATTER, (double)payload_len + 2.0 * total, s);
        }
    }
    if (factored) {
        // factored path: rows first (output T^T, cols x ldh), then the rows of T^T
        if (rows == 1)
            return fdct_axis(ctx, ctx->dense.as<half_bits>(), ldw, src, dir, 1, cols, pn, qn, d_out,
                             1, out_dtype, s, err);
        // the column pass takes the Makhoul fold where it can: the row pass
        // then writes its lines in that pass's column order
        AxisOpts row_opt, col_opt;
        if (makhoul_fold_ok(cols, pm, qm)) {
            row_opt.perm_q = qm;
            row_opt.perm_2p = 2 * pm;
            col_opt.makhoul_fold = true;
        }
        // a spectral payload's row pass takes it too (its pack then only
        // decodes and transposes)
        row_opt.makhoul_fold = src != nullptr && FDCT_FOLD_ROW && makhoul_fold_ok(rows, pn, qn) &&
                               qn % 8 == 0;
        int rc = fdct_axis(ctx, ctx->dense.as<half_bits>(), ldw, src, dir, rows, cols, pn, qn,
                           ctx->tt.p, ldh, HCT_B200_F16, s, err, row_opt);
        if (rc) return rc;
        return fdct_axis(ctx, ctx->tt.as<half_bits>(), ldh, nullptr, dir, cols, rows, pm, qm,
                         d_out, cols, out_dtype, s, err, col_opt);
    }
    const Basis *bw = nullptr, *bh = nullptr;
    int rc = get_basis(ctx, cols, &bw, s, err);
    if (rc) return rc;
    if (rows == 1) {
        // a single row: the column transform of length 1 is the identity
        GemmArgs g{ctx->dense.as<half_bits>(), bw->buf.as<half_bits>(), rows, cols, cols, ldw,
                   bw->ld, d_out, cols, 1, out_dtype, flag};
        int slot = ctx->prof_begin(s);
        CK(launch_umma_gemm(g, s));
        ctx->prof_end(slot, PK_GEMM, 2.0 * rows * cols * cols, s);
        return HCT_B200_OK;
    }
    rc = get_basis(ctx, rows, &bh, s, err);
    if (rc) return rc;
    GemmArgs g1{ctx->dense.as<half_bits>(), bw->buf.as<half_bits>(), rows, cols, cols, ldw,
                bw->ld, ctx->tt.p, ldh, 0, HCT_B200_F16, flag};
    int slot = ctx->prof_begin(s);
    CK(launch_umma_gemm(g1, s));
    ctx->prof_end(slot, PK_GEMM, 2.0 * rows * cols * cols, s);
    GemmArgs g2{bh->buf.as<half_bits>(), ctx->tt.as<half_bits>(), rows, cols, rows, bh->ld, ldh,
                d_out, cols, 1, out_dtype, flag};
    slot = ctx->prof_begin(s);
    CK(launch_umma_gemm(g2, s));
    ctx->prof_end(slot, PK_GEMM, 2.0 * rows * cols * rows, s);
    return HCT_B200_OK;
}

int read_flag(hct_b200_ctx *ctx, cudaStream_t s, hct_b200_error *err) {
    int f = 0;
    CK(cudaMemcpyAsync(&f, ctx->flag.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (f) {
        set_err(err, f, -1, 0, 0, 0, "%s", hct_b200_status_string(f));
        return f;
    }
    return HCT_B200_OK;
}

// First failing block in index order, as HctReader::decompress_all stops there.
int check_block_status(const std::vector<hct_b200_status> &st, hct_b200_error *err) {
    for (size_t i = 0; i < st.size(); i++) {
        const hct_b200_status &s = st[i];
        if (s.code == HCT_B200_OK) continue;
        switch (s.code) {
            case HCT_B200_ERR_UNEXPECTED_EOF:
                set_err(err, s.code, (int)i, s.position, 0, 0, "unexpected EOF after %llu bytes",
                        (unsigned long long)s.position);
                break;
            case HCT_B200_ERR_BUFFER_TOO_SMALL:
                set_err(err, s.code, (int)i, s.position, s.position, s.provided,
                        "buffer too small: need %llu bytes, got %llu",
                        (unsigned long long)s.position, (unsigned long long)s.provided);
                break;
            case HCT_B200_ERR_ZERO_OFFSET:
                set_err(err, s.code, (int)i, s.position, 0, 0,
                        "corrupted data: invalid zero offset");
                break;
            case HCT_B200_ERR_OFFSET_BEYOND:
                set_err(err, s.code, (int)i, s.position, 0, 0,
                        "corrupted data: offset beyond output at offset %llu",
                        (unsigned long long)s.position);
                break;
            default:
                set_err(err, s.code, (int)i, s.position, 0, 0, "block status %d", s.code);
        }
        return s.code;
    }
    return HCT_B200_OK;
}

int lz4_host_call(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len, size_t cap,
                  size_t output_size, uint8_t *out, size_t *written, hct_b200_error *err) {
    clear_err(err);
    if (!ctx || (!in && in_len) || (!out && cap) || !written) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (in_len > 0xffffffffull || cap > 0xffffffffull) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "block larger than 4 GiB");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    int rc = ensure_device(ctx);
    if (rc) { set_err(err, rc, -1, 0, 0, 0, "no CUDA device"); return rc; }
    cudaStream_t s = ctx->stream;
    CK(ctx->io_in.reserve(in_len + 16));
    CK(ctx->io_out.reserve(cap + 16));
    CK(ctx->io_blk.reserve(sizeof(hct_b200_lz4_block)));
    CK(ctx->io_status.reserve(sizeof(hct_b200_status)));
    hct_b200_lz4_block b{0, 0, (uint32_t)in_len, (uint32_t)cap,
                         (uint32_t)std::min<size_t>(output_size, 0xffffffffull), 0};
    if (in_len) CK(cudaMemcpyAsync(ctx->io_in.p, in, in_len, cudaMemcpyHostToDevice, s));
    CK(cudaMemcpyAsync(ctx->io_blk.p, &b, sizeof(b), cudaMemcpyHostToDevice, s));
    CK(launch_lz4_blocks(ctx->io_in.as<uint8_t>(), ctx->io_blk.as<hct_b200_lz4_block>(), 1,
                         ctx->io_out.as<uint8_t>(), ctx->io_status.as<hct_b200_status>(), s));
    std::vector<hct_b200_status> st(1);
    CK(cudaMemcpyAsync(st.data(), ctx->io_status.p, sizeof(hct_b200_status),
                       cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    rc = check_block_status(st, err);
    if (rc) return rc;
    if (st[0].written)
        CK(cudaMemcpy(out, ctx->io_out.p, st[0].written, cudaMemcpyDeviceToHost));
    *written = st[0].written;
    return HCT_B200_OK;
}

}  // namespace

extern "C" {

int hct_b200_abi_version(void) { return HCT_B200_ABI_VERSION; }

const char *hct_b200_status_string(int code) {
    switch (code) {
        case HCT_B200_OK: return "ok";
        case HCT_B200_ERR_UNEXPECTED_EOF: return "unexpected EOF";
        case HCT_B200_ERR_BUFFER_TOO_SMALL: return "buffer too small";
        case HCT_B200_ERR_ZERO_OFFSET: return "corrupted data: invalid zero offset";
        case HCT_B200_ERR_OFFSET_BEYOND: return "corrupted data: offset beyond output";
        case HCT_B200_ERR_INVALID_ARGUMENT: return "invalid argument";
        case HCT_B200_ERR_CORRUPTED: return "corrupted data";
        case HCT_B200_ERR_CHECKSUM: return "checksum mismatch";
        case HCT_B200_ERR_UNSUPPORTED: return "unsupported";
        case HCT_B200_ERR_CUDA: return "CUDA error";
        case HCT_B200_ERR_NO_DEVICE: return "no CUDA device";
        case HCT_B200_ERR_TIMEOUT: return "device wait timed out";
        case HCT_B200_ERR_OUT_OF_MEMORY: return "out of device memory";
        case HCT_B200_ERR_SIZE_MISMATCH: return "payload size does not match the tensor";
        default: return "unknown status";
    }
}

int hct_b200_ctx_create(int device, hct_b200_ctx **out) {
    if (!out) return HCT_B200_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) return HCT_B200_ERR_NO_DEVICE;
    if (device < 0 || device >= n) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (cudaSetDevice(device) != cudaSuccess) return HCT_B200_ERR_NO_DEVICE;
    auto *c = new hct_b200_ctx();
    c->device = device;
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete c;
        return HCT_B200_ERR_CUDA;
    }
    if (cudaStreamCreateWithFlags(&c->side, cudaStreamNonBlocking) != cudaSuccess) {
        cudaStreamDestroy(c->stream);
        delete c;
        return HCT_B200_ERR_CUDA;
    }
    if (c->flag.reserve(sizeof(int)) != cudaSuccess || c->meta.reserve(32) != cudaSuccess) {
        cudaStreamDestroy(c->stream);
        cudaStreamDestroy(c->side);
        delete c;
        return HCT_B200_ERR_OUT_OF_MEMORY;
    }
    cudaMemset(c->flag.p, 0, sizeof(int));
    *out = c;
    return HCT_B200_OK;
}

void hct_b200_ctx_destroy(hct_b200_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    ctx->bases.clear();
    for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->side) cudaStreamDestroy(ctx->side);
    delete ctx;
}

int hct_b200_ctx_reserve(hct_b200_ctx *ctx, uint64_t rows, uint64_t cols) {
    if (!ctx) return HCT_B200_ERR_INVALID_ARGUMENT;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    hct_b200_error e;
    return reserve_spectral(ctx, rows, cols, &e);
}

int hct_b200_ctx_set_idct(hct_b200_ctx *ctx, int mode) {
    if (!ctx || (mode != HCT_B200_IDCT_AUTO && mode != HCT_B200_IDCT_DENSE &&
                 mode != HCT_B200_IDCT_SCATTER))
        return HCT_B200_ERR_INVALID_ARGUMENT;
    ctx->idct_mode = mode;
    return HCT_B200_OK;
}

int hct_b200_ctx_profile(hct_b200_ctx *ctx, int enable) {
    if (!ctx) return HCT_B200_ERR_INVALID_ARGUMENT;
    ctx->profiling = enable != 0;
    ctx->prof.clear();
    ctx->pool_used = 0;
    return HCT_B200_OK;
}

int hct_b200_ctx_profile_read(hct_b200_ctx *ctx, hct_b200_kernel_stats *out, int max_entries,
                              int *count) {
    if (!ctx || !count || (!out && max_entries > 0)) return HCT_B200_ERR_INVALID_ARGUMENT;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    hct_b200_kernel_stats agg[PK_COUNT];
    memset(agg, 0, sizeof(agg));
    for (int k = 0; k < PK_COUNT; k++) snprintf(agg[k].name, sizeof(agg[k].name), "%s", kProfNames[k]);
    for (const ProfRec &r : ctx->prof) {
        if (cudaEventSynchronize(r.b) != cudaSuccess) return HCT_B200_ERR_CUDA;
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, r.a, r.b) != cudaSuccess) return HCT_B200_ERR_CUDA;
        agg[r.kind].launches += 1;
        agg[r.kind].total_ms += ms;
        agg[r.kind].work += r.work;
    }
    int n = 0;
    for (int k = 0; k < PK_COUNT; k++) {
        if (!agg[k].launches) continue;
        if (n < max_entries) out[n] = agg[k];
        n++;
    }
    *count = n;
    return HCT_B200_OK;
}

int hct_b200_lz4_decompress_blocks(const uint8_t *d_src, const hct_b200_lz4_block *d_blocks,
                                   uint32_t num_blocks, uint8_t *d_dst, hct_b200_status *d_status,
                                   uint64_t max_src_len, void *stream) {
    if (num_blocks == 0) return HCT_B200_OK;
    if (!d_src || !d_blocks || !d_dst || !d_status) return HCT_B200_ERR_INVALID_ARGUMENT;
    return cuda_code(launch_lz4_blocks(d_src, d_blocks, num_blocks, d_dst, d_status,
                                       (cudaStream_t)stream, max_src_len));
}

int hct_b200_lz4_decompress_with_size(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len,
                                      size_t output_size, uint8_t *out, size_t *written,
                                      hct_b200_error *err) {
    return lz4_host_call(ctx, in, in_len, output_size, output_size, out, written, err);
}

int hct_b200_lz4_decompress_to(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len, uint8_t *out,
                               size_t out_len, size_t *written, hct_b200_error *err) {
    return lz4_host_call(ctx, in, in_len, out_len, out_len, out, written, err);
}

int hct_b200_dequantize_int4(const uint8_t *d_data, size_t data_len, size_t num_elements,
                             void *d_out, int out_dtype, size_t *written, void *stream) {
    if (!written) return HCT_B200_ERR_INVALID_ARGUMENT;
    *written = 0;
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (num_elements == 0) return HCT_B200_OK;  // quantization.rs:83-85
    const size_t nb = (num_elements + 31) / 32, sb = nb * 2;
    if (data_len < sb) return HCT_B200_OK;       // quantization.rs:90-92
    const size_t n = std::min<size_t>(num_elements, 2 * (data_len - sb));  // :113-115
    if (n && (!d_data || !d_out)) return HCT_B200_ERR_INVALID_ARGUMENT;
    cudaError_t e = launch_dequant_int4(d_data, data_len, n, num_elements, d_out, out_dtype,
                                        nullptr, (cudaStream_t)stream);
    if (e != cudaSuccess) return cuda_code(e);
    *written = n;
    return HCT_B200_OK;
}

int hct_b200_dequantize_int4_batch(const hct_b200_int4_job *jobs, uint32_t num_jobs,
                                   int out_dtype, size_t *written, void *stream) {
    if (num_jobs && (!jobs || !written)) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) return HCT_B200_ERR_INVALID_ARGUMENT;
    std::vector<Int4Job> v;
    v.reserve(num_jobs);
    for (uint32_t i = 0; i < num_jobs; i++) {
        const hct_b200_int4_job &j = jobs[i];
        written[i] = 0;
        if (j.num_elements == 0) continue;                      // quantization.rs:83-85
        const uint64_t sb = (j.num_elements + 31) / 32 * 2;
        if (j.data_len < sb) continue;                          // quantization.rs:90-92
        const uint64_t n = std::min<uint64_t>(j.num_elements, 2 * (j.data_len - sb));  // :113-115
        if (n && (!j.d_data || !j.d_out)) return HCT_B200_ERR_INVALID_ARGUMENT;
        written[i] = n;
        if (n) v.push_back(Int4Job{j.d_data, j.d_out, j.num_elements, n});
    }
    if (v.empty()) return HCT_B200_OK;
    cudaError_t e = launch_dequant_int4_batch(v.data(), (uint32_t)v.size(), out_dtype, nullptr,
                                              (cudaStream_t)stream);
    return e == cudaSuccess ? HCT_B200_OK : cuda_code(e);
}

int hct_b200_dequantize_int4_mp(const uint8_t *d_data, size_t data_len, size_t num_elements,
                                void *d_out, int out_dtype, size_t *written, void *stream) {
    if (!written) return HCT_B200_ERR_INVALID_ARGUMENT;
    *written = 0;
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (num_elements == 0 || data_len == 0) return HCT_B200_OK;  // mixed_precision.rs:490-492
    if (!d_data || !d_out) return HCT_B200_ERR_INVALID_ARGUMENT;
    const cudaStream_t s = (cudaStream_t)stream;
    const size_t esz = out_dtype == HCT_B200_F32 ? 4 : 2;
    const size_t nb = (num_elements + 31) / 32, sb = nb * 2;
    // all zero when the scales do not fit (:497-499), zero past the nibbles (:510-514)
    const size_t n = data_len < sb ? 0 : std::min<size_t>(num_elements, 2 * (data_len - sb));
    if (n) {
        cudaError_t e =
            launch_dequant_int4(d_data, data_len, n, num_elements, d_out, out_dtype, nullptr, s);
        if (e != cudaSuccess) return cuda_code(e);
    }
    if (n < num_elements) {
        cudaError_t e = cudaMemsetAsync(static_cast<uint8_t *>(d_out) + n * esz, 0,
                                        (num_elements - n) * esz, s);
        if (e != cudaSuccess) return cuda_code(e);
    }
    *written = num_elements;
    return HCT_B200_OK;
}

int hct_b200_idct_2d(hct_b200_ctx *ctx, const float *d_in, void *d_out, int out_dtype,
                     size_t width, size_t height, void *stream) {
    if (!ctx || !d_in || !d_out) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (width == 0 || height == 0) return HCT_B200_OK;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    hct_b200_error e, *err = &e;
    clear_err(err);
    cudaStream_t s = (cudaStream_t)stream;
    uint64_t rows = height, cols = width;
    if (cols == 1 && rows > 1) std::swap(rows, cols);  // a column vector: one row transform
    rc = reserve_spectral(ctx, rows, cols, err);
    if (rc) return rc;
    CK(cudaMemsetAsync(ctx->flag.p, 0, sizeof(int), s));
    CK(launch_f32_to_f16_padded(d_in, rows, cols, ctx->dense.as<half_bits>(), round_up(cols, 8), s));
    rc = run_idct(ctx, rows, cols, d_out, out_dtype, s, err);
    if (rc) return rc;
    return read_flag(ctx, s, err);
}

int hct_b200_spectral_q4_decode(hct_b200_ctx *ctx, const uint8_t *d_payload, size_t payload_len,
                                size_t rows_in, size_t cols_in, void *d_out, int out_dtype,
                                void *stream) {
    if (!ctx || !d_payload || !d_out) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (((uintptr_t)d_payload & 15u) != 0) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (rows_in == 0 || cols_in == 0) return HCT_B200_OK;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    hct_b200_error e, *err = &e;
    clear_err(err);
    cudaStream_t s = (cudaStream_t)stream;
    uint64_t rows = rows_in, cols = cols_in;
    if (cols == 1 && rows > 1) std::swap(rows, cols);
    const uint64_t total = rows * cols;
    if (payload_len < (total + 7) / 8) return HCT_B200_ERR_SIZE_MISMATCH;
    rc = reserve_spectral(ctx, rows, cols, err);
    if (rc) return rc;
    CK(cudaMemsetAsync(ctx->flag.p, 0, sizeof(int), s));
    rc = run_idct(ctx, rows, cols, d_out, out_dtype, s, err, d_payload, payload_len);
    if (rc) return rc;
    return read_flag(ctx, s, err);
}

// ---- Zstandard --------------------------------------------------------------
// zstd::decode_all on the GPU (zstd_decode.cu): the host only moves bytes and
// reads statuses.

namespace {

// Skips one zstd frame's blocks and checksum (header already read); false
// when they run past the end.
bool zstd_skip_blocks(const uint8_t *src, size_t len, size_t *p, bool cksum) {
    for (;;) {
        if (len - *p < 3) return false;
        const uint32_t bh = (uint32_t)src[*p] | ((uint32_t)src[*p + 1] << 8) |
                            ((uint32_t)src[*p + 2] << 16);
        *p += 3;
        const uint32_t type = (bh >> 1) & 3, bsize = bh >> 3;
        if (type == 3) return false;
        const size_t body = type == 1 ? 1 : bsize;
        if (len - *p < body) return false;
        *p += body;
        if (bh & 1) break;
    }
    if (cksum) {
        if (len - *p < 4) return false;
        *p += 4;
    }
    return true;
}

// Content size of every frame (RFC 8878 3.1.1.1.4): HCT_B200_OK with the sum,
// HCT_B200_ERR_UNSUPPORTED if a frame does not record it.
int zstd_sizes(const uint8_t *src, size_t len, uint64_t *total) {
    size_t ip = 0;
    uint64_t sum = 0;
    bool known = true;
    while (ip < len) {
        if (len - ip < 4) return HCT_B200_ERR_CORRUPTED;
        const uint32_t magic = rd32(src + ip);
        if ((magic & 0xFFFFFFF0u) == 0x184D2A50u) {
            if (len - ip < 8) return HCT_B200_ERR_CORRUPTED;
            const uint64_t sz = rd32(src + ip + 4);
            if (len - ip - 8 < sz) return HCT_B200_ERR_CORRUPTED;
            ip += 8 + sz;
            continue;
        }
        if (magic != 0xFD2FB528u || len - ip < 5) return HCT_B200_ERR_CORRUPTED;
        size_t p = ip + 4;
        const int fhd = src[p++];
        const int fcs_flag = fhd >> 6, single = (fhd >> 5) & 1, dflag = fhd & 3;
        const int dbytes = dflag == 0 ? 0 : (dflag == 1 ? 1 : (dflag == 2 ? 2 : 4));
        const int fbytes = fcs_flag == 0 ? (single ? 1 : 0) : (fcs_flag == 1 ? 2 : (fcs_flag == 2 ? 4 : 8));
        const size_t hl = (size_t)(single ? 0 : 1) + dbytes + fbytes;
        if (len - p < hl) return HCT_B200_ERR_CORRUPTED;
        p += (single ? 0 : 1) + dbytes;
        uint64_t fcs = 0;
        for (int i = 0; i < fbytes; i++) fcs |= (uint64_t)src[p + i] << (8 * i);
        if (fbytes == 2) fcs += 256;
        p += fbytes;
        if (fbytes == 0) known = false;
        sum += fcs;
        if (!zstd_skip_blocks(src, len, &p, (fhd >> 2) & 1)) return HCT_B200_ERR_CORRUPTED;
        ip = p;
    }
    *total = sum;
    return known ? HCT_B200_OK : HCT_B200_ERR_UNSUPPORTED;
}

// Host bytes in -> host bytes out on the context's stream; capacity cap.
// Returns the decode status code (the error filled for non-OK codes).
int zstd_host_call(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len, size_t cap,
                   std::vector<uint8_t> *out, hct_b200_error *err) {
    int rc = ensure_device(ctx);
    if (rc) { set_err(err, rc, -1, 0, 0, 0, "no CUDA device"); return rc; }
    const cudaStream_t s = ctx->stream;
    CK(ctx->zsrc.reserve(in_len + 16));
    CK(ctx->zdst.reserve(cap + 16));
    CK(ctx->zjob.reserve(sizeof(hct_b200_zstd_job)));
    CK(ctx->zstatus.reserve(sizeof(hct_b200_status)));
    CK(ctx->zscratch.reserve(zstd_scratch_bytes(1)));
    if (in_len) CK(cudaMemcpyAsync(ctx->zsrc.p, in, in_len, cudaMemcpyHostToDevice, s));
    const hct_b200_zstd_job job{0, in_len, 0, cap};
    CK(cudaMemcpyAsync(ctx->zjob.p, &job, sizeof(job), cudaMemcpyHostToDevice, s));
    CK(launch_zstd_decode(ctx->zsrc.as<uint8_t>(), ctx->zjob.as<hct_b200_zstd_job>(), 1,
                          ctx->zdst.as<uint8_t>(), ctx->zstatus.as<hct_b200_status>(),
                          ctx->zscratch.as<uint8_t>(), s));
    hct_b200_status st{};
    CK(cudaMemcpyAsync(&st, ctx->zstatus.p, sizeof(st), cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    if (st.code != HCT_B200_OK) {
        set_err(err, st.code, -1, st.position, st.code == HCT_B200_ERR_BUFFER_TOO_SMALL ? cap + 1 : 0,
                cap, "zstd: %s at input offset %llu",
                st.code == HCT_B200_ERR_BUFFER_TOO_SMALL
                    ? "output larger than the buffer"
                    : (st.code == HCT_B200_ERR_CHECKSUM
                           ? "content checksum mismatch"
                           : (st.code == HCT_B200_ERR_UNSUPPORTED ? "frame needs a dictionary"
                                                                  : "corrupted frame")),
                (unsigned long long)st.position);
        return st.code;
    }
    out->resize(st.written);
    if (st.written)
        CK(cudaMemcpy(out->data(), ctx->zdst.p, st.written, cudaMemcpyDeviceToHost));
    return HCT_B200_OK;
}

// zstd::decode_all: the content size when every frame records it, else
// growing capacities (the 4x guess and doubling of the reference's
// Decompressor::decompress, up to 4 GiB).
int zstd_decode_all(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len,
                    std::vector<uint8_t> *out, hct_b200_error *err) {
    uint64_t known = 0;
    size_t cap = zstd_sizes(in, in_len, &known) == HCT_B200_OK ? (size_t)known
                                                               : std::max<size_t>(in_len * 4, 4096);
    for (;;) {
        const int rc = zstd_host_call(ctx, in, in_len, cap, out, err);
        if (rc != HCT_B200_ERR_BUFFER_TOO_SMALL || cap >= (4ull << 30)) return rc;
        cap *= 2;
    }
}

}  // namespace

int hct_b200_zstd_content_size(const uint8_t *in, size_t in_len, uint64_t *size) {
    if (!size || (!in && in_len)) return HCT_B200_ERR_INVALID_ARGUMENT;
    *size = 0;
    return zstd_sizes(in, in_len, size);
}

int hct_b200_zstd_decompress_jobs(hct_b200_ctx *ctx, const uint8_t *d_src,
                                  const hct_b200_zstd_job *d_jobs, uint32_t n, uint8_t *d_dst,
                                  hct_b200_status *d_status, void *stream) {
    if (!ctx || (n && (!d_src || !d_jobs || !d_dst || !d_status))) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (n == 0) return HCT_B200_OK;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    cudaError_t e = ctx->zscratch.reserve(zstd_scratch_bytes(n));
    if (e != cudaSuccess) return cuda_code(e);
    e = launch_zstd_decode(d_src, d_jobs, n, d_dst, d_status, ctx->zscratch.as<uint8_t>(),
                           (cudaStream_t)stream);
    return cuda_code(e);
}

int hct_b200_zstd_decompress(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len, uint8_t *out,
                             size_t out_cap, size_t *written, hct_b200_error *err) {
    clear_err(err);
    if (!ctx || !written || (!in && in_len) || (!out && out_cap)) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    *written = 0;
    std::vector<uint8_t> res;
    const int rc = zstd_host_call(ctx, in, in_len, out_cap, &res, err);
    if (rc) return rc;
    if (!res.empty()) memcpy(out, res.data(), res.size());
    *written = res.size();
    return HCT_B200_OK;
}

// ---- V3 fragment container -----------------------------------------------
// haagenti-cuda's GpuDecompressor::parse_hct_fragments + reconstruct_coefficients
// (crates/haagenti-cuda/src/decompress.rs:322-438) and the reference's C
// hct_decode (ref/c/hct_decoder.h:322-394).  Fragments are accepted as the C
// decoder accepts them: parsing stops at a header or fragment that runs past
// the data, and a fragment is skipped when its coefficient count, bitmap or
// values do not fit (the Rust parser raises on a fragment past the end and
// reads as many values as the bytes hold; on well-formed data both agree).

int hct_b200_v3_open(hct_b200_ctx *ctx, const uint8_t *data, size_t len, uint64_t rows,
                     uint64_t cols, hct_b200_v3 **out, hct_b200_error *err) {
    clear_err(err);
    if (!ctx || !out || (!data && len)) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    // zstd wrapper (decompress.rs:296-319): decoded on the GPU; data that
    // does not decode is parsed as it is
    std::vector<uint8_t> unwrapped;
    if (len >= 4 && rd32(data) == 0xFD2FB528u) {
        hct_b200_error zerr;
        if (zstd_decode_all(ctx, data, len, &unwrapped, &zerr) == HCT_B200_OK) {
            data = unwrapped.data();
            len = unwrapped.size();
        }
        clear_err(err);
    }
    if (len < 2) {  // decompress.rs:323-325
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "HCT data too short");
        return HCT_B200_ERR_CORRUPTED;
    }
    auto v = std::make_unique<hct_b200_v3>();
    v->ctx = ctx;
    v->rows = rows;
    v->cols = cols;
    if (v->cols == 1 && v->rows > 1) std::swap(v->rows, v->cols);
    const uint64_t total = rows * cols;
    const uint64_t bmb = (total + 7) / 8;
    struct Src {
        size_t bm, vals;
        uint64_t n;
    };
    std::vector<Src> src;
    if (total) {
        const uint32_t nfrag = rd16(data);
        size_t pos = 2;
        for (uint32_t f = 0; f < nfrag && pos < len; f++) {
            if (pos + 16 > len) break;
            const uint64_t dlen = rd32(data + pos + 12);
            pos += 16;
            if (pos + dlen > len) break;
            const size_t fd = pos;
            pos += dlen;
            if (dlen < 4) continue;
            const uint64_t n = rd32(data + fd);
            if (4 + bmb > dlen || 4 + bmb + 2 * n > dlen) continue;
            src.push_back(Src{fd + 4, fd + 4 + bmb, n});
        }
    }
    // device layout: per fragment its bitmap then its values, each 16-byte aligned
    size_t bytes = 0;
    for (const Src &f : src) {
        hct_b200_v3::Frag g;
        g.bm_off = bytes;
        bytes += round_up(bmb, 16);
        g.vals_off = bytes;
        bytes += round_up(2 * f.n, 16);
        g.nvals = f.n;
        v->frags.push_back(g);
    }
    int rc = ensure_device(ctx);
    if (rc) { set_err(err, rc, -1, 0, 0, 0, "no CUDA device"); return rc; }
    cudaStream_t s = ctx->stream;
    CK(v->d_data.reserve(bytes + 64));
    for (size_t i = 0; i < src.size(); i++) {
        CK(cudaMemcpyAsync(v->d_data.as<uint8_t>() + v->frags[i].bm_off, data + src[i].bm, bmb,
                           cudaMemcpyHostToDevice, s));
        if (src[i].n)
            CK(cudaMemcpyAsync(v->d_data.as<uint8_t>() + v->frags[i].vals_off, data + src[i].vals,
                               2 * src[i].n, cudaMemcpyHostToDevice, s));
    }
    if (total) {
        rc = reserve_spectral(ctx, v->rows, v->cols, err);
        if (rc) return rc;
    }
    CK(cudaStreamSynchronize(s));
    *out = v.release();
    return HCT_B200_OK;
}

int hct_b200_v3_num_fragments(const hct_b200_v3 *v) { return v ? (int)v->frags.size() : 0; }

int hct_b200_v3_decode(hct_b200_v3 *v, void *d_out, int out_dtype, void *stream,
                       hct_b200_error *err) {
    clear_err(err);
    if (!v || !d_out) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "bad output dtype");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    hct_b200_ctx *ctx = v->ctx;
    const uint64_t rows = v->rows, cols = v->cols, total = rows * cols;
    if (total == 0) return HCT_B200_OK;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    const cudaStream_t s = (cudaStream_t)stream;
    const uint64_t ldw = round_up(cols, 8);
    int *flag = ctx->flag.as<int>();
    CK(cudaMemsetAsync(flag, 0, sizeof(int), s));
    if (v->frags.empty()) CK(cudaMemsetAsync(ctx->dense.p, 0, rows * ldw * 2, s));
    for (size_t i = 0; i < v->frags.size(); i++) {
        const hct_b200_v3::Frag &f = v->frags[i];
        int slot = ctx->prof_begin(s);
        CK(launch_v3_scatter(v->d_data.as<uint8_t>() + f.bm_off, total, cols,
                             reinterpret_cast<const uint16_t *>(v->d_data.as<uint8_t>() + f.vals_off),
                             f.nvals, ctx->chunk.as<uint32_t>(), ctx->meta.as<uint64_t>(), flag,
                             ctx->dense.as<half_bits>(), ldw, i == 0, s));
        ctx->prof_end(slot, PK_SCATTER, (double)((total + 7) / 8) + 2.0 * f.nvals + 2.0 * total, s);
    }
    rc = run_idct(ctx, rows, cols, d_out, out_dtype, s, err);
    if (rc) return rc;
    return read_flag(ctx, s, err);
}

void hct_b200_v3_close(hct_b200_v3 *v) {
    if (!v) return;
    cudaSetDevice(v->ctx->device);
    delete v;
}

int hct_b200_hct_v3_decode(hct_b200_ctx *ctx, const uint8_t *data, size_t len, uint64_t rows,
                           uint64_t cols, void *d_out, int out_dtype, void *stream,
                           hct_b200_error *err) {
    hct_b200_v3 *v = nullptr;
    int rc = hct_b200_v3_open(ctx, data, len, rows, cols, &v, err);
    if (rc) return rc;
    rc = hct_b200_v3_decode(v, d_out, out_dtype, stream, err);
    hct_b200_v3_close(v);
    return rc;
}

// ---- HoloTensor -------------------------------------------------------------
// HoloTensorReader (crates/haagenti-hct/src/holotensor.rs:1935-2192) and the
// SV03 part of SpectralDecoder (:840-1051).  The container is parsed on the
// host; every fragment's values are uploaded once; a decode scatters the
// first k fragments into the dense fp16 coefficient matrix (holo.cu) and runs
// the IDCT of idct_gemm.cu / fdct.cu on it.

namespace {

constexpr uint32_t HOLO_VERSION = 1;                  // holotensor.rs:50
constexpr uint16_t HOLO_FLAG_HEADER_CHECKSUM = 0x0001;  // :53
constexpr uint16_t HOLO_FLAG_FRAGMENT_CHECKSUMS = 0x0002;  // :56
constexpr size_t HOLO_HEADER_SIZE = 96;               // HoloTensorHeader::BASE_SIZE, :442
constexpr size_t HOLO_ENTRY_SIZE = 24;                // FragmentIndexEntry::SIZE, :349
constexpr uint32_t SV03_MAGIC = 0x33305653;           // :794

// QualityCurve::predict (holotensor.rs:199-220) in f32, one rounding per
// operation as the Rust code has.
float holo_predict(const hct_b200_holo_info &h, uint32_t k, uint32_t n) {
    if (n == 0) return 0.0f;
    if (k >= n) return 1.0f;
    if (k < h.min_fragments) return 0.0f;
    const float x = (float)k / (float)n;
    float result = 0.0f, xp = 1.0f;
    for (int i = 0; i < 4; i++) {
        volatile float t = h.quality_curve[i] * xp;
        result = result + t;
        volatile float nx = xp * x;
        xp = nx;
    }
    return result < 0.0f ? 0.0f : (result > 1.0f ? 1.0f : result);
}

uint32_t holo_total(const hct_b200_holo *h) {
    return h->hdr.inline_format ? 1u : (uint32_t)h->hdr.total_fragments;
}

}  // namespace

int hct_b200_holo_open(hct_b200_ctx *ctx, const uint8_t *file, size_t len, hct_b200_holo **out,
                       hct_b200_error *err) {
    clear_err(err);
    if (!ctx || !out || (!file && len)) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    // HoloTensorHeader::from_bytes (holotensor.rs:571-656)
    if (len < HOLO_HEADER_SIZE) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "failed to read header");
        return HCT_B200_ERR_CORRUPTED;
    }
    if (memcmp(file, "HTNS", 4) != 0) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "invalid magic bytes");
        return HCT_B200_ERR_CORRUPTED;
    }
    const uint32_t version = rd32(file + 4);
    if (version != HOLO_VERSION) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "unsupported version: %u", version);
        return HCT_B200_ERR_CORRUPTED;
    }
    const uint16_t flags = rd16(file + 10);
    Xxh3Fn xxh = xxh3_fn();
    if ((flags & (HOLO_FLAG_HEADER_CHECKSUM | HOLO_FLAG_FRAGMENT_CHECKSUMS)) && !xxh) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "XXH3 (libxxhash) unavailable");
        return HCT_B200_ERR_UNSUPPORTED;
    }
    if ((flags & HOLO_FLAG_HEADER_CHECKSUM) && rd64(file + 88) != xxh(file, 88)) {
        set_err(err, HCT_B200_ERR_CHECKSUM, -1, 0, 0, 0, "header checksum mismatch");
        return HCT_B200_ERR_CHECKSUM;
    }
    if (file[8] > 2 || file[9] > 1 || file[32] > 4) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "unknown %s: %u",
                file[8] > 2 ? "encoding" : (file[9] > 1 ? "algorithm" : "dtype"),
                file[8] > 2 ? file[8] : (file[9] > 1 ? file[9] : file[32]));
        return HCT_B200_ERR_CORRUPTED;
    }
    auto h = std::make_unique<hct_b200_holo>();
    h->ctx = ctx;
    hct_b200_holo_info &hd = h->hdr;
    hd.encoding = file[8];
    hd.compression = file[9];
    hd.flags = flags;
    hd.total_fragments = rd16(file + 12);
    hd.min_fragments = rd16(file + 14);
    hd.original_size = rd64(file + 16);
    hd.seed = rd64(file + 24);
    hd.dtype = file[32];
    hd.ndim = file[33];
    if (34 + 8 * (size_t)hd.ndim > HOLO_HEADER_SIZE) {  // the shape would run past the header
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "shape of %u dimensions", hd.ndim);
        return HCT_B200_ERR_CORRUPTED;
    }
    for (int i = 0; i < hd.ndim; i++) hd.shape[i] = rd64(file + 34 + 8 * i);
    for (int i = 0; i < 4; i++) {
        const uint32_t bits = rd32(file + 66 + 4 * i);
        memcpy(&hd.quality_curve[i], &bits, 4);
    }
    // HoloTensorDecoder::new's 2-D view (holotensor.rs:1732-1744)
    uint64_t rows = 1, cols = 1;
    if (hd.ndim == 1) {
        cols = hd.shape[0];
    } else if (hd.ndim == 2) {
        rows = hd.shape[0];
        cols = hd.shape[1];
    } else if (hd.ndim > 2) {
        rows = hd.shape[0];
        for (int i = 1; i < hd.ndim; i++) {
            if (hd.shape[i] && cols > UINT64_MAX / hd.shape[i]) {
                set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "shape overflows");
                return HCT_B200_ERR_CORRUPTED;
            }
            cols *= hd.shape[i];
        }
    }
    if (cols && rows > UINT64_MAX / cols) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "shape overflows");
        return HCT_B200_ERR_CORRUPTED;
    }
    hd.rows = rows;
    hd.cols = cols;
    h->rows = rows;
    h->cols = cols;
    if (h->cols == 1 && h->rows > 1) std::swap(h->rows, h->cols);
    // fragment index (HoloTensorReader::new, holotensor.rs:1955-2003)
    const size_t nidx = hd.total_fragments;
    size_t data_offset = HOLO_HEADER_SIZE + nidx * HOLO_ENTRY_SIZE;
    if (len < data_offset) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "failed to read fragment index");
        return HCT_B200_ERR_CORRUPTED;
    }
    struct Entry {
        uint16_t index, flags;
        uint32_t offset, csize, usize;
        uint64_t checksum;
        size_t base;  // file offset the entry's offset is relative to
    };
    std::vector<Entry> entries;
    for (size_t i = 0; i < nidx; i++) {
        const uint8_t *e = file + HOLO_HEADER_SIZE + i * HOLO_ENTRY_SIZE;
        entries.push_back(Entry{rd16(e), rd16(e + 2), rd32(e + 4), rd32(e + 8), rd32(e + 12),
                                rd64(e + 16), data_offset});
    }
    if (nidx == 0 && len >= data_offset + HOLO_ENTRY_SIZE) {
        const uint8_t *e = file + data_offset;
        const uint32_t csize = rd32(e + 8);
        if (rd16(e) == 0 && csize > 0 && csize < 1000000000u) {
            entries.push_back(Entry{0, rd16(e + 2), rd32(e + 4), csize, rd32(e + 12), rd64(e + 16),
                                    data_offset + HOLO_ENTRY_SIZE});
            hd.inline_format = 1;
        }
    }
    // each fragment as read_fragment + add_fragment would see it
    struct Src {
        size_t frag;  // index into h->frags
        size_t at;    // file offset of its values (SV03) or of its zstd frames
        uint64_t n;   // values, or compressed bytes
        uint64_t cap; // zstd: output capacity
    };
    std::vector<Src> plain, packed;
    // SV03 header of fragment bytes d (n of them) into f
    auto classify = [](hct_b200_holo::Frag &f, const uint8_t *d, uint64_t n) {
        if (n < 8) {
            f.kind = hct_b200_holo::SHORT;
        } else if (rd32(d) != SV03_MAGIC) {
            f.kind = hct_b200_holo::LEGACY;
        } else if (n < 20) {
            f.kind = hct_b200_holo::V3_SHORT;
        } else {  // add_fragment_v3 (holotensor.rs:979-1015)
            f.kind = hct_b200_holo::SV03;
            f.num_coeffs = rd32(d + 4);
            f.F = rd32(d + 8);
            f.start = rd32(d + 12);
            const uint64_t nv = (n - 20) / 4;
            if (f.start >= f.num_coeffs) f.count = 0;
            else if (f.F == 0) f.count = nv;
            else f.count = std::min<uint64_t>(nv, (f.num_coeffs - f.start + (uint64_t)f.F - 1) / f.F);
        }
    };
    for (const Entry &e : entries) {
        hct_b200_holo::Frag f;
        f.index = e.index;
        const size_t at = e.base + e.offset;
        if (at > len || e.csize > len - at) {
            f.kind = hct_b200_holo::PAST_END;
        } else {
            const uint8_t *d = file + at;
            if (flags & HOLO_FLAG_FRAGMENT_CHECKSUMS) f.checksum_ok = xxh(d, e.csize) == e.checksum;
            if (e.flags & 1) {  // zstd (holotensor.rs:2081-2091), decoded on the GPU below
                uint64_t fcs = 0;
                uint64_t cap = zstd_sizes(d, e.csize, &fcs) == HCT_B200_OK ? fcs : 0;
                cap = std::max<uint64_t>(cap, e.usize);
                if (cap == 0) cap = 4ull * e.csize + 4096;
                packed.push_back(Src{h->frags.size(), at, e.csize, cap});
            } else {
                classify(f, d, e.csize);
                if (f.kind == hct_b200_holo::SV03) plain.push_back(Src{h->frags.size(), at + 20, f.count, 0});
            }
        }
        h->frags.push_back(f);
    }
    int rc = ensure_device(ctx);
    if (rc) { set_err(err, rc, -1, 0, 0, 0, "no CUDA device"); return rc; }
    cudaStream_t s = ctx->stream;
    // device layout: the plain fragments' values, then one 16-byte aligned
    // region per zstd fragment for its decoded bytes (values at +20 bytes)
    for (int attempt = 0;; attempt++) {
        uint64_t total_vals = 0;
        for (const Src &p : plain) {
            h->frags[p.frag].dev_off = total_vals;
            total_vals += round_up(p.n, 4);
        }
        std::vector<uint64_t> region(packed.size());
        uint64_t zbytes = 0, zin = 0;
        for (size_t i = 0; i < packed.size(); i++) {
            region[i] = 4 * total_vals + zbytes;
            zbytes += round_up(packed[i].cap, 16);
            zin += round_up(packed[i].n, 16);
        }
        CK(h->d_vals.reserve(total_vals * 4 + zbytes + 64));
        for (const Src &p : plain)
            if (p.n)
                CK(cudaMemcpyAsync(h->d_vals.as<float>() + h->frags[p.frag].dev_off, file + p.at,
                                   4 * p.n, cudaMemcpyHostToDevice, s));
        if (packed.empty()) break;
        std::vector<hct_b200_zstd_job> jobs(packed.size());
        CK(ctx->zsrc.reserve(zin + 16));
        uint64_t off = 0;
        for (size_t i = 0; i < packed.size(); i++) {
            CK(cudaMemcpyAsync(ctx->zsrc.as<uint8_t>() + off, file + packed[i].at, packed[i].n,
                               cudaMemcpyHostToDevice, s));
            jobs[i] = hct_b200_zstd_job{off, packed[i].n, region[i], packed[i].cap};
            off += round_up(packed[i].n, 16);
        }
        CK(ctx->zjob.reserve(jobs.size() * sizeof(hct_b200_zstd_job)));
        CK(ctx->zstatus.reserve(jobs.size() * sizeof(hct_b200_status)));
        CK(ctx->zscratch.reserve(zstd_scratch_bytes((uint32_t)jobs.size())));
        CK(cudaMemcpyAsync(ctx->zjob.p, jobs.data(), jobs.size() * sizeof(hct_b200_zstd_job),
                           cudaMemcpyHostToDevice, s));
        CK(launch_zstd_decode(ctx->zsrc.as<uint8_t>(), ctx->zjob.as<hct_b200_zstd_job>(),
                              (uint32_t)jobs.size(), h->d_vals.as<uint8_t>(),
                              ctx->zstatus.as<hct_b200_status>(), ctx->zscratch.as<uint8_t>(), s));
        std::vector<hct_b200_status> st(jobs.size());
        CK(cudaMemcpyAsync(st.data(), ctx->zstatus.p, st.size() * sizeof(hct_b200_status),
                           cudaMemcpyDeviceToHost, s));
        CK(cudaStreamSynchronize(s));
        bool grow = false;
        for (size_t i = 0; i < packed.size(); i++)
            if (st[i].code == HCT_B200_ERR_BUFFER_TOO_SMALL && packed[i].cap < (4ull << 30)) {
                packed[i].cap *= 2;  // decode_all grows its output until the frames fit
                grow = true;
            }
        if (grow && attempt < 40) continue;
        // the decoded fragments' SV03 headers
        for (size_t i = 0; i < packed.size(); i++) {
            hct_b200_holo::Frag &f = h->frags[packed[i].frag];
            if (st[i].code != HCT_B200_OK) {
                f.kind = hct_b200_holo::ZSTD_BAD;
                continue;
            }
            uint8_t head[20] = {0};
            const uint64_t w = st[i].written;
            if (w) CK(cudaMemcpy(head, h->d_vals.as<uint8_t>() + region[i], std::min<uint64_t>(w, 20),
                                 cudaMemcpyDeviceToHost));
            classify(f, head, w);
            f.dev_off = (region[i] + 20) / 4;
        }
        break;
    }
    if (h->rows && h->cols) {
        rc = reserve_spectral(ctx, h->rows, h->cols, err);
        if (rc) return rc;
    }
    CK(cudaStreamSynchronize(s));
    *out = h.release();
    return HCT_B200_OK;
}

int hct_b200_holo_header(const hct_b200_holo *h, hct_b200_holo_info *out) {
    if (!h || !out) return HCT_B200_ERR_INVALID_ARGUMENT;
    *out = h->hdr;
    return HCT_B200_OK;
}

int hct_b200_holo_total_fragments(const hct_b200_holo *h) { return h ? (int)holo_total(h) : 0; }

float hct_b200_holo_predict_quality(const hct_b200_holo *h, uint32_t k) {
    if (!h) return 0.0f;
    const uint32_t n = holo_total(h);
    return holo_predict(h->hdr, k, n ? n : 1);
}

uint32_t hct_b200_holo_fragments_for_quality(const hct_b200_holo *h, float target) {
    if (!h) return 0;
    const uint32_t total = holo_total(h);
    for (uint32_t i = 0; i < total; i++)
        if (holo_predict(h->hdr, i + 1, total ? total : 1) >= target) return i + 1;
    return total;
}

int hct_b200_holo_decode(hct_b200_holo *h, uint32_t num_fragments, void *d_out, int out_dtype,
                         void *stream, float *quality, hct_b200_error *err) {
    clear_err(err);
    if (!h || !d_out) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "bad output dtype");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (h->hdr.encoding != 0) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0,
                "HoloTensor encoding %u (only the spectral encoding is decoded)", h->hdr.encoding);
        return HCT_B200_ERR_UNSUPPORTED;
    }
    // read_fragment(i) for i < k, then add_fragment (holotensor.rs:2039-2098, 840-858)
    std::vector<const hct_b200_holo::Frag *> used;
    for (uint32_t i = 0; i < num_fragments; i++) {
        const hct_b200_holo::Frag *f = nullptr;
        if (h->hdr.inline_format) {
            if (i != 0) {
                set_err(err, HCT_B200_ERR_CORRUPTED, (int)i, 0, 0, 0,
                        "inline format only has fragment 0, requested %u", i);
                return HCT_B200_ERR_CORRUPTED;
            }
            f = &h->frags[0];
        } else {
            for (const auto &g : h->frags)
                if (g.index == i) { f = &g; break; }
            if (!f) {
                set_err(err, HCT_B200_ERR_CORRUPTED, (int)i, 0, 0, 0, "fragment %u not found", i);
                return HCT_B200_ERR_CORRUPTED;
            }
        }
        const char *why = nullptr;
        int code = HCT_B200_ERR_CORRUPTED;
        if (f->kind == hct_b200_holo::PAST_END) why = "failed to read fragment data";
        else if (!f->checksum_ok) { why = "fragment checksum mismatch"; code = HCT_B200_ERR_CHECKSUM; }
        else if (f->kind == hct_b200_holo::ZSTD_BAD) why = "failed to decompress fragment";
        else if (f->kind == hct_b200_holo::SHORT) why = "fragment too short";
        else if (f->kind == hct_b200_holo::V3_SHORT) why = "V3 fragment too short";
        else if (f->kind == hct_b200_holo::LEGACY) { why = "V1/V2 spectral fragment layout"; code = HCT_B200_ERR_UNSUPPORTED; }
        if (why) {
            set_err(err, code, (int)i, 0, 0, 0, "fragment %u: %s", i, why);
            return code;
        }
        used.push_back(f);
    }
    if (used.empty()) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "no fragments loaded");
        return HCT_B200_ERR_CORRUPTED;
    }
    hct_b200_ctx *ctx = h->ctx;
    const uint64_t rows = h->rows, cols = h->cols, n = rows * cols;
    if (n == 0) {
        if (quality) *quality = NAN;  // 0 / 0, as the reference's f32 division
        return HCT_B200_OK;
    }
    int rc = ensure_device(ctx);
    if (rc) return rc;
    const cudaStream_t s = (cudaStream_t)stream;
    const uint64_t ldw = round_up(cols, 8);
    half_bits *dense = ctx->dense.as<half_bits>();
    // One stride and distinct residues: the output-major interleave.
    const uint32_t F = used[0]->F;
    bool interleave = F > 0 && F <= (1u << 22) && n < (1ull << 40);
    std::vector<Sv03Residue> res;
    if (interleave) {
        res.assign(F, Sv03Residue{0, 0, 0});
        std::vector<uint8_t> seen(F, 0);
        for (const auto *f : used) {
            if (f->F != F || seen[f->start % F]) { interleave = false; break; }
            seen[f->start % F] = 1;
            res[f->start % F] = Sv03Residue{f->dev_off, f->start / F, f->count};
        }
    }
    uint64_t covered = 0;
    int *flag = ctx->flag.as<int>();
    CK(cudaMemsetAsync(flag, 0, sizeof(int), s));
    int slot = ctx->prof_begin(s);
    if (interleave) {
        for (const auto *f : used)
            if (f->start < n) covered += std::min<uint64_t>(f->count, (n - f->start + F - 1) / F);
        CK(h->d_res.reserve(sizeof(Sv03Residue) * F));
        CK(cudaMemcpyAsync(h->d_res.p, res.data(), sizeof(Sv03Residue) * F,
                           cudaMemcpyHostToDevice, s));
        CK(launch_sv03_interleave(h->d_vals.as<float>(), h->d_res.as<Sv03Residue>(), F, rows, cols,
                                  dense, ldw, s));
    } else {
        // positions in load order, later fragments over earlier ones
        std::vector<bool> set(n, false);
        CK(cudaMemsetAsync(dense, 0, rows * ldw * 2, s));
        for (const auto *f : used) {
            CK(launch_sv03_scatter(h->d_vals.as<float>() + f->dev_off, f->count, f->start, f->F,
                                   n, cols, dense, ldw, s));
            for (uint64_t j = 0; j < f->count; j++) {
                if (f->F == 0 && j + 1 != f->count) continue;
                const uint64_t p = f->start + (uint64_t)f->F * j;
                if (p < n && !set[p]) { set[p] = true; covered++; }
            }
        }
    }
    uint64_t vals_read = 0;
    for (const auto *f : used) vals_read += f->count;
    ctx->prof_end(slot, PK_SCATTER, 4.0 * (double)vals_read + 2.0 * (double)n, s);
    if (quality) *quality = (float)covered / (float)n;
    rc = run_idct(ctx, rows, cols, d_out, out_dtype, s, err);
    if (rc) return rc;
    return read_flag(ctx, s, err);
}

void hct_b200_holo_close(hct_b200_holo *h) {
    if (!h) return;
    cudaSetDevice(h->ctx->device);
    delete h;
}

// ---- reader ----------------------------------------------------------------

int hct_b200_reader_open(hct_b200_ctx *ctx, const uint8_t *file, size_t file_len,
                         int validate_checksums, hct_b200_reader **out, hct_b200_error *err) {
    clear_err(err);
    if (!ctx || !file || !out) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    // header (HctHeader::from_bytes, tensor.rs:332-374)
    if (file_len < 64) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0,
                "hct error: failed to read header: file shorter than 64 bytes");
        return HCT_B200_ERR_CORRUPTED;
    }
    if (memcmp(file, "HCTN", 4) != 0) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "corrupted data: invalid HCT magic");
        return HCT_B200_ERR_CORRUPTED;
    }
    auto r = std::make_unique<hct_b200_reader>();
    hct_b200_header &h = r->hdr;
    h.version = rd32(file + 4);
    if (h.version > 2) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0,
                "corrupted data: unsupported HCT version: %u (max: 2)", h.version);
        return HCT_B200_ERR_CORRUPTED;
    }
    h.algorithm = file[8];
    h.dtype = file[9];
    if (h.algorithm > 1) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "corrupted data: unknown algorithm: %u",
                h.algorithm);
        return HCT_B200_ERR_CORRUPTED;
    }
    if (h.dtype > 4) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "corrupted data: unknown dtype: %u",
                h.dtype);
        return HCT_B200_ERR_CORRUPTED;
    }
    h.flags = rd16(file + 10);
    h.original_size = rd64(file + 12);
    h.compressed_size = rd64(file + 20);
    h.block_size = rd32(file + 28);
    h.num_blocks = rd32(file + 32);
    h.rank = file[36];
    for (uint32_t i = 0; i < std::min<uint32_t>(h.rank, 4); i++) h.shape[i] = rd64(file + 37 + 8 * i);
    const bool v2 = h.version >= 2;
    // v2 header checksum (HctReaderV2::new, tensor.rs:853-865)
    if (v2 && (h.flags & FLAG_HEADER_CHECKSUM)) {
        Xxh3Fn x = xxh3_fn();
        if (!x) {
            set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "XXH3 (libxxhash) unavailable");
            return HCT_B200_ERR_UNSUPPORTED;
        }
        const uint64_t stored = rd64(file + 56), computed = x(file, 56);
        if (stored != computed) {
            set_err(err, HCT_B200_ERR_CHECKSUM, -1, 0, 0, 0,
                    "corrupted data: header checksum mismatch: expected %016llx, got %016llx",
                    (unsigned long long)stored, (unsigned long long)computed);
            return HCT_B200_ERR_CHECKSUM;
        }
    }
    size_t pos = 64;
    if (v2 && (h.flags & FLAG_QUANTIZATION)) {
        if (file_len < pos + 8) {
            set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0,
                    "hct error: failed to read quantization");
            return HCT_B200_ERR_CORRUPTED;
        }
        memcpy(h.quant_meta, file + pos, 8);
        h.has_quant_meta = 1;
        pos += 8;
    }
    const bool sums = v2 && (h.flags & FLAG_BLOCK_CHECKSUMS);
    const size_t ent = sums ? 16 : 8;
    const uint32_t nb = h.num_blocks;
    if ((file_len - pos) / ent < nb) {
        set_err(err, HCT_B200_ERR_CORRUPTED, -1, 0, 0, 0, "hct error: failed to read block index");
        return HCT_B200_ERR_CORRUPTED;
    }
    r->offsets.resize(nb);
    r->sizes.resize(nb);
    r->checksums.assign(nb, 0);
    for (uint32_t i = 0; i < nb; i++) {
        const uint8_t *e = file + pos + (size_t)i * ent;
        r->offsets[i] = rd32(e);
        r->sizes[i] = rd32(e + 4);
        r->max_block = std::max<uint64_t>(r->max_block, r->sizes[i]);
        if (sums) r->checksums[i] = rd64(e + 8);
    }
    pos += (size_t)nb * ent;
    r->data_offset = pos;
    r->data_len = file_len - pos;
    for (uint32_t i = 0; i < nb; i++) {
        if ((uint64_t)r->offsets[i] + r->sizes[i] > r->data_len) {
            set_err(err, HCT_B200_ERR_CORRUPTED, (int)i, 0, 0, 0,
                    "hct error: failed to read block %u", i);
            return HCT_B200_ERR_CORRUPTED;
        }
    }
    // per-block expected sizes (tensor.rs:494-500)
    r->expected.resize(nb);
    if (nb) {
        const uint64_t full = (uint64_t)(nb - 1) * h.block_size;
        if (h.original_size < full || h.original_size - full > 0xffffffffull) {
            set_err(err, HCT_B200_ERR_CORRUPTED, nb - 1, 0, 0, 0,
                    "corrupted data: original size inconsistent with the block count");
            return HCT_B200_ERR_CORRUPTED;
        }
        for (uint32_t i = 0; i + 1 < nb; i++) r->expected[i] = h.block_size;
        r->expected[nb - 1] = (uint32_t)(h.original_size - full);
    }
    if (validate_checksums && sums) {
        Xxh3Fn x = xxh3_fn();
        if (!x) {
            set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "XXH3 (libxxhash) unavailable");
            return HCT_B200_ERR_UNSUPPORTED;
        }
        for (uint32_t i = 0; i < nb; i++) {
            if (r->checksums[i] == 0) continue;  // tensor.rs:957
            const uint64_t c = x(file + pos + r->offsets[i], r->sizes[i]);
            if (c != r->checksums[i]) {
                set_err(err, HCT_B200_ERR_CHECKSUM, (int)i, 0, 0, 0,
                        "corrupted data: block %u checksum mismatch: expected %016llx, got %016llx",
                        i, (unsigned long long)r->checksums[i], (unsigned long long)c);
                return HCT_B200_ERR_CHECKSUM;
            }
        }
    }
    // tensor geometry for the decode
    uint64_t rows = 1, cols = 1;
    if (h.rank == 1) {
        cols = h.shape[0];
    } else if (h.rank >= 2) {
        for (uint32_t i = 0; i + 1 < std::min<uint32_t>(h.rank, 4); i++) rows *= h.shape[i];
        cols = h.shape[std::min<uint32_t>(h.rank, 4) - 1];
    } else {
        cols = 0;
    }
    r->rows = rows;
    r->cols = cols;
    r->spectral = (h.flags & HCT_B200_FLAG_SPECTRAL_Q4) != 0;
    r->ctx = ctx;

    int rc = ensure_device(ctx);
    if (rc) { set_err(err, rc, -1, 0, 0, 0, "no CUDA device"); return rc; }
    cudaStream_t s = ctx->stream;
    CK(r->d_data.reserve(r->data_len + 64));
    CK(r->d_blocks.reserve((size_t)std::max<uint32_t>(nb, 1) * sizeof(hct_b200_lz4_block)));
    CK(r->d_status.reserve((size_t)std::max<uint32_t>(nb, 1) * sizeof(hct_b200_status)));
    CK(cudaMallocHost(&r->h_status, (size_t)std::max<uint32_t>(nb, 1) * sizeof(hct_b200_status)));
    CK(cudaMallocHost(&r->h_flag, sizeof(int)));
    CK(cudaEventCreateWithFlags(&r->done, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&r->uploaded, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&r->data_free, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&r->front_done, cudaEventDisableTiming));
    CK(cudaEventCreateWithFlags(&r->back_done, cudaEventDisableTiming));
    CK(r->d_payload.reserve(h.original_size + 64));
    CK(r->d_meta.reserve(4 * sizeof(uint64_t)));
    CK(r->d_flag.reserve(sizeof(int)));
    if (h.dtype == 4 && r->spectral)
        CK(r->d_chunk.reserve(rank_dir_words(rows * cols) * sizeof(uint32_t)));
    std::vector<hct_b200_lz4_block> blocks(nb);
    for (uint32_t i = 0; i < nb; i++) {
        blocks[i].src_off = r->offsets[i];
        blocks[i].dst_off = (uint64_t)i * h.block_size;
        blocks[i].src_len = r->sizes[i];
        blocks[i].dst_cap = r->expected[i];
        blocks[i].out_size = r->expected[i];
        blocks[i].reserved = 0;
    }
    if (r->data_len)
        CK(cudaMemcpyAsync(r->d_data.p, file + pos, r->data_len, cudaMemcpyHostToDevice, s));
    if (nb)
        CK(cudaMemcpyAsync(r->d_blocks.p, blocks.data(), nb * sizeof(hct_b200_lz4_block),
                           cudaMemcpyHostToDevice, s));
    if (h.dtype == 4 && r->spectral) {
        // the back end's matrices live in the context (the payload in the reader)
        uint64_t rr = rows, cc = cols;
        if (cc == 1 && rr > 1) std::swap(rr, cc);
        rc = reserve_spectral(ctx, rr, cc, err);
        if (rc) return rc;
    }
    CK(cudaStreamSynchronize(s));
    *out = r.release();
    return HCT_B200_OK;
}

int hct_b200_reader_upload(hct_b200_reader *r, const uint8_t *file, size_t file_len, void *stream) {
    if (!r || !file) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (file_len != r->data_offset + r->data_len) return HCT_B200_ERR_SIZE_MISMATCH;
    const cudaStream_t s = (cudaStream_t)stream;
    hct_b200_error *err = nullptr;  // this entry point reports the status code only
    int rc = ensure_device(r->ctx);
    if (rc) return rc;
    if (r->read_pending) CK(cudaStreamWaitEvent(s, r->data_free, 0));
    CK(cudaMemcpyAsync(r->d_data.p, file + r->data_offset, r->data_len, cudaMemcpyHostToDevice, s));
    CK(cudaEventRecord(r->uploaded, s));
    r->upload_pending = true;
    return HCT_B200_OK;
}

int hct_b200_reader_header(const hct_b200_reader *r, hct_b200_header *out) {
    if (!r || !out) return HCT_B200_ERR_INVALID_ARGUMENT;
    *out = r->hdr;
    return HCT_B200_OK;
}

uint32_t hct_b200_reader_num_blocks(const hct_b200_reader *r) { return r ? r->hdr.num_blocks : 0; }

namespace {

// LZ4 stage into dst; returns the total written after the reference's
// truncate-and-concatenate rule (compacting on the device if a block is short).
int reader_lz4(hct_b200_reader *r, uint8_t *d_dst, size_t cap, size_t *written, cudaStream_t s,
               hct_b200_error *err) {
    const uint32_t nb = r->hdr.num_blocks;
    if (cap < r->hdr.original_size) {
        set_err(err, HCT_B200_ERR_BUFFER_TOO_SMALL, -1, r->hdr.original_size, r->hdr.original_size,
                cap, "buffer too small: need %llu bytes, got %zu",
                (unsigned long long)r->hdr.original_size, cap);
        return HCT_B200_ERR_BUFFER_TOO_SMALL;
    }
    *written = 0;
    if (nb == 0) return HCT_B200_OK;
    if (r->back_pending) CK(cudaStreamWaitEvent(s, r->back_done, 0));  // d_status in use
    CK(r->before_read(s));
    int slot = r->ctx->prof_begin(s);
    CK(launch_lz4_blocks(r->d_data.as<uint8_t>(), r->d_blocks.as<hct_b200_lz4_block>(), nb, d_dst,
                         r->d_status.as<hct_b200_status>(), s, r->max_block));
    r->ctx->prof_end(slot, PK_LZ4, (double)r->hdr.compressed_size + (double)r->hdr.original_size, s);
    CK(r->after_read(s));
    std::vector<hct_b200_status> st(nb);
    CK(cudaMemcpyAsync(st.data(), r->d_status.p, nb * sizeof(hct_b200_status),
                       cudaMemcpyDeviceToHost, s));
    CK(cudaStreamSynchronize(s));
    int rc = check_block_status(st, err);
    if (rc) return rc;
    uint64_t total = 0;
    bool compact = false;
    for (uint32_t i = 0; i < nb; i++) {
        if (compact && st[i].written)
            CK(cudaMemcpyAsync(d_dst + total, d_dst + (uint64_t)i * r->hdr.block_size,
                               st[i].written, cudaMemcpyDeviceToDevice, s));
        if (st[i].written != r->expected[i]) compact = true;
        total += st[i].written;
    }
    if (compact) CK(cudaStreamSynchronize(s));
    *written = total;
    return HCT_B200_OK;
}

}  // namespace

int hct_b200_reader_decompress_all(hct_b200_reader *r, uint8_t *d_out, size_t out_cap,
                                   size_t *written, void *stream, hct_b200_error *err) {
    clear_err(err);
    if (!r || (!d_out && r->hdr.original_size) || !written) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (r->hdr.algorithm != 0) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "only LZ4 containers are decoded");
        return HCT_B200_ERR_UNSUPPORTED;
    }
    int rc = ensure_device(r->ctx);
    if (rc) return rc;
    return reader_lz4(r, d_out, out_cap, written, (cudaStream_t)stream, err);
}

int hct_b200_reader_decode(hct_b200_reader *r, void *d_out, int out_dtype, void *stream,
                           hct_b200_error *err) {
    clear_err(err);
    if (!r || !d_out) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "bad output dtype");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (r->hdr.algorithm != 0) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "only LZ4 containers are decoded");
        return HCT_B200_ERR_UNSUPPORTED;
    }
    if (r->hdr.dtype != 4) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "only I4 tensors are decoded");
        return HCT_B200_ERR_UNSUPPORTED;
    }
    int rc = hct_b200_reader_decode_async(r, d_out, out_dtype, stream, err);
    if (rc) return rc;
    return hct_b200_reader_wait(r, err);
}

// The whole decode is enqueued with no host synchronisation, in two parts:
//  - front end on the context's side stream: LZ4 into the reader's payload
//    (per-block statuses) and, for a spectral tensor decoded through the
//    fused row pack, the payload's rank directory;
//  - back end on `stream`, after the front end: INT4 dequantisation or the
//    IDCT, then the statuses and the device flag copied to pinned host
//    memory.
// Consecutive decodes of different readers thus overlap one tensor's front
// end with the previous tensor's back end; a reader's next front end waits
// for its previous back end.  hct_b200_reader_wait then reports exactly what
// hct_b200_reader_decode would have (the output is undefined when it reports
// an error).
int hct_b200_reader_decode_async(hct_b200_reader *r, void *d_out, int out_dtype, void *stream,
                                 hct_b200_error *err) {
    clear_err(err);
    if (!r || !d_out) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "null argument");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (out_dtype < HCT_B200_F32 || out_dtype > HCT_B200_BF16) {
        set_err(err, HCT_B200_ERR_INVALID_ARGUMENT, -1, 0, 0, 0, "bad output dtype");
        return HCT_B200_ERR_INVALID_ARGUMENT;
    }
    if (r->hdr.algorithm != 0) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "only LZ4 containers are decoded");
        return HCT_B200_ERR_UNSUPPORTED;
    }
    if (r->hdr.dtype != 4) {
        set_err(err, HCT_B200_ERR_UNSUPPORTED, -1, 0, 0, 0, "only I4 tensors are decoded");
        return HCT_B200_ERR_UNSUPPORTED;
    }
    hct_b200_ctx *ctx = r->ctx;
    int rc = ensure_device(ctx);
    if (rc) return rc;
    const cudaStream_t s = (cudaStream_t)stream, fs = ctx->side;
    const uint32_t nb = r->hdr.num_blocks;
    const uint64_t total = r->rows * r->cols;
    uint64_t rows = r->rows, cols = r->cols;
    if (cols == 1 && rows > 1) std::swap(rows, cols);
    uint8_t *payload = r->d_payload.as<uint8_t>();
    const size_t written = r->hdr.original_size;  // verified against the statuses in _wait
    RankDir dir{r->d_chunk.as<uint32_t>(), r->d_meta.as<uint64_t>(), r->d_flag.as<int>(), false};

    // ---- front end (side stream)
    if (r->back_pending) CK(cudaStreamWaitEvent(fs, r->back_done, 0));
    CK(cudaMemsetAsync(r->d_flag.p, 0, sizeof(int), fs));
    if (nb) {
        CK(r->before_read(fs));
        int slot = ctx->prof_begin(fs);
        CK(launch_lz4_blocks(r->d_data.as<uint8_t>(), r->d_blocks.as<hct_b200_lz4_block>(), nb,
                             payload, r->d_status.as<hct_b200_status>(), fs, r->max_block));
        ctx->prof_end(slot, PK_LZ4, (double)r->hdr.compressed_size + (double)r->hdr.original_size,
                      fs);
        CK(r->after_read(fs));
    }
    if (total && r->spectral && spectral_fused(ctx, rows, cols)) {
        int slot = ctx->prof_begin(fs);
        CK(launch_spectral_rank(payload, written, total, dir.chunk, dir.meta, dir.flag, fs));
        ctx->prof_end(slot, PK_RANK, (double)((total + 7) / 8), fs);
        dir.ranked = true;
    }
    CK(cudaEventRecord(r->front_done, fs));

    // ---- back end (caller's stream)
    CK(cudaStreamWaitEvent(s, r->front_done, 0));
    r->pending_elems = 0;
    if (total && !r->spectral) {
        // plain INT4 weights (examples/safetensors_to_int4_hct.rs:241-284)
        size_t n = 0;
        int slot = ctx->prof_begin(s);
        rc = hct_b200_dequantize_int4(payload, written, total, d_out, out_dtype, &n, s);
        ctx->prof_end(slot, PK_DEQUANT, (double)written + (out_dtype == HCT_B200_F32 ? 4.0 : 2.0) * n,
                      s);
        if (rc) return rc;
        r->pending_elems = n;
    } else if (total) {
        rc = run_idct(ctx, rows, cols, d_out, out_dtype, s, err, payload, written, &dir);
        if (rc) return rc;
    }
    if (nb)
        CK(cudaMemcpyAsync(r->h_status, r->d_status.p, nb * sizeof(hct_b200_status),
                           cudaMemcpyDeviceToHost, s));
    CK(cudaMemcpyAsync(r->h_flag, r->d_flag.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    CK(cudaEventRecord(r->done, s));
    CK(cudaEventRecord(r->back_done, s));
    r->back_pending = true;
    r->pending = true;
    return HCT_B200_OK;
}

int hct_b200_reader_wait(hct_b200_reader *r, hct_b200_error *err) {
    clear_err(err);
    if (!r) return HCT_B200_ERR_INVALID_ARGUMENT;
    if (!r->pending) return HCT_B200_OK;
    r->pending = false;
    CK(cudaEventSynchronize(r->done));
    const uint32_t nb = r->hdr.num_blocks;
    std::vector<hct_b200_status> st(r->h_status, r->h_status + nb);
    int rc = check_block_status(st, err);
    if (rc) return rc;
    uint64_t got = 0;
    for (uint32_t i = 0; i < nb; i++) got += st[i].written;
    if (got != r->hdr.original_size) {
        set_err(err, HCT_B200_ERR_SIZE_MISMATCH, -1, 0, r->hdr.original_size, got,
                "decompressed payload holds %llu of %llu bytes", (unsigned long long)got,
                (unsigned long long)r->hdr.original_size);
        return HCT_B200_ERR_SIZE_MISMATCH;
    }
    const uint64_t total = r->rows * r->cols;
    if (!r->spectral && r->pending_elems != total) {
        set_err(err, HCT_B200_ERR_SIZE_MISMATCH, -1, 0, total, r->pending_elems,
                "INT4 payload holds %llu of %llu elements", (unsigned long long)r->pending_elems,
                (unsigned long long)total);
        return HCT_B200_ERR_SIZE_MISMATCH;
    }
    if (*r->h_flag) {
        set_err(err, *r->h_flag, -1, 0, 0, 0, "%s", hct_b200_status_string(*r->h_flag));
        return *r->h_flag;
    }
    return HCT_B200_OK;
}

void hct_b200_reader_close(hct_b200_reader *r) {
    if (!r) return;
    cudaSetDevice(r->ctx->device);
    delete r;
}

}  // extern "C"
