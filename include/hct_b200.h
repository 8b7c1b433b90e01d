/*
 * hct_b200.h -- C ABI of the B200 HCT weight-decode library (libhct_b200.so).
 *
 * Drop-in boundary for haagenti's HCT decode path: LZ4 block decompression
 * -> INT4 dequantisation with per-block FP16 scales -> inverse-DCT spectral
 * reconstruction.  Each entry point names the reference interface it
 * replaces (paths relative to the haagenti repository root).
 *
 * Conventions
 *  - Plain pointers and sizes only.  `d_` pointers are CUDA device pointers,
 *    other buffers are host memory.  `stream` is a cudaStream_t (NULL = the
 *    legacy default stream).
 *  - Every function returns an hct_b200 status code (0 = success).  Codes
 *    1..4 map 1:1 onto haagenti_core::Error variants raised by
 *    crates/haagenti-lz4/src/block.rs:261-366.
 *  - Kernels never trap: a corrupt block yields a per-block status, a device
 *    wait that does not complete within its bound yields HCT_B200_ERR_TIMEOUT.
 *  - There is no CPU fallback: without a usable CUDA device every entry
 *    point returns HCT_B200_ERR_NO_DEVICE.
 */
#ifndef HCT_B200_H
#define HCT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HCT_B200_ABI_VERSION 2

/* ---- status codes ------------------------------------------------------ */
enum {
    HCT_B200_OK = 0,
    HCT_B200_ERR_UNEXPECTED_EOF = 1,     /* Error::UnexpectedEof{bytes_read}      (block.rs:279,294,315,331) */
    HCT_B200_ERR_BUFFER_TOO_SMALL = 2,   /* Error::BufferTooSmall{required,provided} (block.rs:297,346)    */
    HCT_B200_ERR_ZERO_OFFSET = 3,        /* Error::corrupted("invalid zero offset")   (block.rs:321)        */
    HCT_B200_ERR_OFFSET_BEYOND = 4,      /* Error::corrupted_at("offset beyond output", pos) (block.rs:324) */
    HCT_B200_ERR_INVALID_ARGUMENT = 16,
    HCT_B200_ERR_CORRUPTED = 17,         /* container-level Error::CorruptedData (tensor.rs:334-374, 463-468) */
    HCT_B200_ERR_CHECKSUM = 18,          /* XXH3 mismatch (tensor.rs:857-865, 966-973)                       */
    HCT_B200_ERR_UNSUPPORTED = 19,       /* e.g. a zstd frame that needs a dictionary                      */
    HCT_B200_ERR_CUDA = 20,
    HCT_B200_ERR_NO_DEVICE = 21,
    HCT_B200_ERR_TIMEOUT = 22,           /* a bounded device-side wait expired                              */
    HCT_B200_ERR_OUT_OF_MEMORY = 23,
    HCT_B200_ERR_SIZE_MISMATCH = 24      /* decoded payload shorter/longer than the tensor needs           */
};

/* Output element types; values equal haagenti_hct::DType tags (tensor.rs:98-105). */
enum { HCT_B200_F32 = 0, HCT_B200_F16 = 1, HCT_B200_BF16 = 2 };

/* One independent LZ4 block: decompress_block(src[src_off..+src_len],
 * &mut dst[dst_off..+dst_cap], out_size).  dst_cap is `output.len()`,
 * out_size is `output_size` (block.rs:261). */
typedef struct {
    uint64_t src_off;
    uint64_t dst_off;
    uint32_t src_len;
    uint32_t dst_cap;
    uint32_t out_size;
    uint32_t reserved;
} hct_b200_lz4_block;

/* Per-block result.  position = bytes_read (EOF), required (BufferTooSmall)
 * or output_pos (offset errors); provided = `provided` of BufferTooSmall;
 * written = bytes produced (the Ok(usize) value on success). */
typedef struct {
    int32_t code;
    int32_t reserved;
    uint64_t position;
    uint64_t provided;
    uint64_t written;
} hct_b200_status;

/* Host-side error report for the higher-level calls. */
typedef struct {
    int32_t code;
    int32_t block;        /* failing block index, -1 if not block-specific */
    uint64_t position;
    uint64_t required;
    uint64_t provided;
    char message[192];
} hct_b200_error;

/* HctHeader (tensor.rs:275-292) plus version and the v2 extras. */
typedef struct {
    uint32_t version;
    uint8_t algorithm;
    uint8_t dtype;
    uint16_t flags;
    uint64_t original_size;
    uint64_t compressed_size;
    uint32_t block_size;
    uint32_t num_blocks;
    uint32_t rank;
    uint32_t reserved;
    uint64_t shape[4];
    uint8_t quant_meta[8]; /* QuantizationMetadata bytes when FLAG_QUANTIZATION */
    uint32_t has_quant_meta;
    uint32_t reserved2;
} hct_b200_header;

/* Flag of this library's composite spectral payload (bitmap ++ INT4 of the
 * retained DCT coefficients).  Not a reference flag: the reference defines
 * 0x0001..0x0010 (tensor.rs:53-69). */
#define HCT_B200_FLAG_SPECTRAL_Q4 0x0100u

typedef struct hct_b200_ctx hct_b200_ctx;
typedef struct hct_b200_reader hct_b200_reader;
typedef struct hct_b200_v3 hct_b200_v3;
typedef struct hct_b200_holo hct_b200_holo;

/* ---- context ------------------------------------------------------------
 * One context per device owns the scratch memory, the cached DCT bases and
 * the TMA descriptors.  Replaces GpuContext (crates/haagenti-cuda/src/lib.rs:89-230).
 * Calls on one context must be serialised by the caller (as GpuContext). */
int hct_b200_ctx_create(int device, hct_b200_ctx **out);
void hct_b200_ctx_destroy(hct_b200_ctx *ctx);
/* Grow the context's scratch so that decoding a rows x cols spectral
 * tensor needs no further allocation. */
int hct_b200_ctx_reserve(hct_b200_ctx *ctx, uint64_t rows, uint64_t cols);
const char *hct_b200_status_string(int code);
int hct_b200_abi_version(void);

/* How the context computes the IDCT.  AUTO (default) uses the factored
 * transform (a Makhoul pack pass and two short tcgen05 DFT contractions per
 * axis; O(n) tensor-core FLOPs per element, HBM-bound) whenever both axis
 * lengths factor as 2*P*Q with P, Q multiples of 4 up to 128, and the dense
 * contraction against the full DCT basis otherwise; DENSE always uses the
 * dense contraction.  Both compute haagenti_core::dct::idct_2d
 * (crates/haagenti-core/src/dct.rs:311-337). */
/* SCATTER: the factored transform, but a spectral payload is first scattered
 * into a dense fp16 matrix instead of being decoded inside the row pack. */
enum { HCT_B200_IDCT_AUTO = 0, HCT_B200_IDCT_DENSE = 1, HCT_B200_IDCT_SCATTER = 2 };
int hct_b200_ctx_set_idct(hct_b200_ctx *ctx, int mode);

/* Per-kernel timing of the context's own launches, for roofline reports.
 * With profiling enabled every kernel launch made through the context is
 * bracketed by CUDA events recorded on its launch stream; _read synchronises
 * those events and returns one entry per kernel kind that ran
 * (lz4_decode_blocks, spectral_scatter, umma_gemm, dequant_int4,
 * makhoul_pack, dft_stage1, spectral_rank, spectral_pack, dft_stage2).
 * `work` is the algorithmic work summed over launches: FLOPs (2*M*N*K) for
 * umma_gemm, bytes read + written for the others.  No reference counterpart (the reference keeps
 * ad-hoc DecompressStats, crates/haagenti-cuda/src/decompress.rs:55-94). */
typedef struct {
    char name[32];
    uint64_t launches;
    double total_ms;
    double work;
} hct_b200_kernel_stats;
int hct_b200_ctx_profile(hct_b200_ctx *ctx, int enable); /* enable/disable; clears records */
int hct_b200_ctx_profile_read(hct_b200_ctx *ctx, hct_b200_kernel_stats *out, int max_entries,
                              int *count);

/* ---- LZ4 ----------------------------------------------------------------
 * Batched form of block::decompress_block (crates/haagenti-lz4/src/block.rs:261),
 * one warp per independent block.  Results are exact: byte-for-byte output and
 * the same error variant/position as the reference for every block.
 * max_src_len is an upper bound of the blocks' src_len when the caller knows
 * one, else 0; a bound up to the LZ4 bound of a 16 KiB block (16464) lets the
 * kernel stage each compressed block in shared memory (the layout the HCT
 * container uses).  A wrong bound never affects results, only the variant.
 * Stream-ordered; d_status is written when the kernel completes. */
int hct_b200_lz4_decompress_blocks(const uint8_t *d_src, const hct_b200_lz4_block *d_blocks,
                                   uint32_t num_blocks, uint8_t *d_dst,
                                   hct_b200_status *d_status, uint64_t max_src_len,
                                   void *stream);

/* Lz4Decompressor::decompress_with_size (crates/haagenti-lz4/src/decompress.rs:63-68)
 * on host buffers: `out` must hold output_size bytes; *written = truncated length. */
int hct_b200_lz4_decompress_with_size(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len,
                                      size_t output_size, uint8_t *out, size_t *written,
                                      hct_b200_error *err);

/* Lz4Decompressor::decompress_to (decompress.rs:59-61): output.len() == out_len. */
int hct_b200_lz4_decompress_to(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len, uint8_t *out,
                               size_t out_len, size_t *written, hct_b200_error *err);

/* Writer side (host CPU; produces the blocks the decoder consumes):
 * block::compress_block (crates/haagenti-lz4/src/block.rs:73-147) and
 * max_compressed_size (block.rs:370-373).  _chunks compresses block_size
 * chunks as HctWriter::compress_data does (crates/haagenti-hct/src/tensor.rs:
 * 556-562), chunk i written at out + i*out_stride, its length in lens[i]. */
size_t hct_b200_lz4_max_compressed_size(size_t n);
int hct_b200_lz4_compress_block(const uint8_t *in, size_t in_len, uint8_t *out, size_t out_cap,
                                size_t *out_len);
int hct_b200_lz4_compress_chunks(const uint8_t *in, size_t in_len, size_t block_size,
                                 uint8_t *out, size_t out_stride, uint32_t *lens);
/* quantize_int4 (crates/haagenti/src/testing/quantization.rs:30-70): `out`
 * holds ceil(n/32)*2 + ceil(n/2) bytes (scales first, low nibble first). */
int hct_b200_quantize_int4(const float *w, size_t n, uint8_t *out);
/* mixed_precision.rs:448-486: the same layout with each scale stored as the
 * round-to-nearest-even f16 (half::f16::from_f32). */
int hct_b200_quantize_int4_mp(const float *w, size_t n, uint8_t *out);
/* Retention step of CompressiveSpectralEncoder::encode_2d (crates/haagenti/src/
 * compressive.rs:140-172): the k largest |c| (ties to the lower index) as an
 * LSB-first bitmap of ceil(n/8) bytes and their values in index order. */
int hct_b200_spectral_select(const float *coeffs, size_t n, size_t k, uint8_t *bitmap,
                             float *values, size_t *count);

/* ---- INT4 ---------------------------------------------------------------
 * haagenti::testing::dequantize_int4 (crates/haagenti/src/testing/quantization.rs:82-131):
 * out[i] = f32(nibble_i - 8) * f32(scale[i/32]); layout [ceil(n/32) f16 LE scales]
 * [ceil(n/2) nibble bytes, low nibble first].  *written follows the reference's
 * short-input rules (0 if the scales do not fit, fewer than n if the nibbles run
 * out) and is known on return without a device sync.  F32 output is bit-exact;
 * F16/BF16 outputs are the round-to-nearest-even of that f32 value. */
int hct_b200_dequantize_int4(const uint8_t *d_data, size_t data_len, size_t num_elements,
                             void *d_out, int out_dtype, size_t *written, void *stream);
/* Many dequantize_int4 calls in few launches (no single reference
 * counterpart: each job is haagenti::testing::dequantize_int4,
 * crates/haagenti/src/testing/quantization.rs:82-131, with the same short-input
 * rules; written[i] receives job i's element count).  For a loader decoding a
 * model of plain INT4 tensors (examples/safetensors_to_int4_hct.rs) without a
 * launch per tensor.  Stream-ordered, no host synchronisation. */
typedef struct {
    const uint8_t *d_data;   /* f16 scales, then nibbles (the quantize_int4 layout) */
    uint64_t data_len;
    uint64_t num_elements;
    void *d_out;             /* num_elements of out_dtype */
} hct_b200_int4_job;
int hct_b200_dequantize_int4_batch(const hct_b200_int4_job *jobs, uint32_t num_jobs,
                                   int out_dtype, size_t *written, void *stream);
/* The private INT4 pair of haagenti::mixed_precision (crates/haagenti/src/
 * mixed_precision.rs:489-539): the same values, but always num_elements of
 * them -- all zero when the scales do not fit, zero past the end of the
 * nibbles -- and nothing for num_elements == 0 or empty data
 * (*written = 0). */
int hct_b200_dequantize_int4_mp(const uint8_t *d_data, size_t data_len, size_t num_elements,
                                void *d_out, int out_dtype, size_t *written, void *stream);

/* ---- IDCT ---------------------------------------------------------------
 * haagenti_core::dct::idct_2d (crates/haagenti-core/src/dct.rs:311-337) and
 * GpuDctContext::idct_2d (crates/haagenti-cuda/src/dct_gpu.rs:1404-1412):
 * orthonormal 2-D DCT-III of a row-major height x width f32 matrix, as two
 * dense contractions against the DCT basis on tcgen05 tensor cores (fp16
 * operands, fp32 accumulation in TMEM). */
int hct_b200_idct_2d(hct_b200_ctx *ctx, const float *d_in, void *d_out, int out_dtype,
                     size_t width, size_t height, void *stream);

/* Decode an already LZ4-decompressed spectral payload held on the device
 * (bitmap ++ quantize_int4(values)), rows x cols, into d_out.  The INT4
 * dequantisation and bitmap scatter run on the GPU and feed the two IDCT
 * contractions (CompressiveSpectralDecoder::reconstruct, crates/haagenti/src/
 * compressive.rs:732-752, with INT4 values in place of FP16).  d_payload must
 * be 16-byte aligned (the kernels read the bitmap in 64-bit and 128-bit
 * words); an unaligned pointer returns HCT_B200_ERR_INVALID_ARGUMENT. */
int hct_b200_spectral_q4_decode(hct_b200_ctx *ctx, const uint8_t *d_payload, size_t payload_len,
                                size_t rows, size_t cols, void *d_out, int out_dtype,
                                void *stream);

/* Allocation-free variant of hct_b200_spectral_q4_decode for callers that
 * cannot allocate device memory while they decode (a serving runtime whose
 * allocator owns all of HBM, or code that must not trigger the device-wide
 * synchronisation of cudaMalloc/cudaFree).  It has no counterpart in the
 * reference.  It takes no context and allocates nothing: its scratch is one
 * fixed 32 MiB device array inside the library (held on every device that
 * uses the library until the process exits), so rows and cols must each be
 * <= 2048; larger tensors return HCT_B200_ERR_INVALID_ARGUMENT.
 * It decodes on the calling thread's current device: d_payload (16-byte
 * aligned), d_out and stream must belong to that device.  The first call on
 * a device looks up that array's device address and keeps it for the life of
 * the process; make that first call before any stream capture begins, and
 * do not call it again on a device after cudaDeviceReset there.  All calls
 * share the array: calls whose GPU work overlaps race and must be serialised
 * by the caller.  Each call copies the device-side status to host memory and
 * synchronises `stream` before it returns. */
int hct_b200_spectral_q4_decode_noalloc(const uint8_t *d_payload, size_t payload_len, size_t rows,
                                        size_t cols, void *d_out, int out_dtype, void *stream);

/* ---- HCT V3 fragments (bitmap + fp16 coefficients) ----------------------
 * GpuDecompressor::decompress for HCT V3 data (crates/haagenti-cuda/src/
 * decompress.rs:322-438: parse_hct_fragments, reconstruct_coefficients, IDCT)
 * and the reference's C hct_decode (ref/c/hct_decoder.h:322-394):
 *   [num_fragments u16], per fragment [index u16][flags u16][checksum u64]
 *   [data_len u32][num_coefficients u32][bitmap ceil(rows*cols/8)][f16 values]
 * Each fragment writes its values, in index order, at its bitmap's set bits
 * (later fragments over earlier ones, the rest zero), then the orthonormal
 * 2-D DCT-III of rows x cols.  Fragments are accepted as hct_decode accepts
 * them (a fragment whose bitmap or values do not fit is skipped; parsing
 * stops at a fragment past the end).  open parses the headers on the host
 * and uploads each fragment's bitmap and values once; decode is
 * stream-ordered and synchronises once to read the device flag.
 * hct_b200_hct_v3_decode is open + decode + close.  Data that starts with
 * the zstd magic is zstd-decoded first (on the GPU; decompress.rs:296-319,
 * where data that does not decode is parsed as it is).  Fewer than 2 bytes
 * of data is HCT_B200_ERR_CORRUPTED ("HCT data too short",
 * decompress.rs:323). */
int hct_b200_v3_open(hct_b200_ctx *ctx, const uint8_t *data, size_t len, uint64_t rows,
                     uint64_t cols, hct_b200_v3 **out, hct_b200_error *err);
int hct_b200_v3_num_fragments(const hct_b200_v3 *v);
int hct_b200_v3_decode(hct_b200_v3 *v, void *d_out, int out_dtype, void *stream,
                       hct_b200_error *err);
void hct_b200_v3_close(hct_b200_v3 *v);
int hct_b200_hct_v3_decode(hct_b200_ctx *ctx, const uint8_t *data, size_t len, uint64_t rows,
                           uint64_t cols, void *d_out, int out_dtype, void *stream,
                           hct_b200_error *err);

/* ---- Zstandard ------------------------------------------------------------
 * zstd::decode_all as the reference calls it (crates/haagenti-hct/src/
 * holotensor.rs:2081-2091 for fragments with entry flag bit 0,
 * crates/haagenti-cuda/src/decompress.rs:296-319 for zstd-wrapped HCT
 * data): every frame of a job's input in turn (RFC 8878; skippable frames
 * skipped, content checksums and frame content sizes verified), their
 * contents concatenated.  Frames that need a dictionary are
 * HCT_B200_ERR_UNSUPPORTED.  Valid frames decode to the same bytes as
 * libzstd; on corrupted input this decoder reports an error wherever libzstd
 * does and in some cases where libzstd's fast Huffman path returns data
 * (every literal stream must be consumed exactly).
 * The reference's ZstdGpuPipeline (crates/haagenti-cuda/src/zstd_gpu.rs:
 * 348-402: decompress, decompress_batch, decompress_to_gpu) maps onto these
 * three calls (it decodes on the CPU; this decoder runs on the GPU).
 * jobs: several jobs per launch.  A job holding one frame whose blocks
 * regenerate the encoder's block size (min(128 KiB, window), the last one the
 * rest of the content size) is decoded block-parallel, a warp per block;
 * any other job by one warp.  Per-job status
 * {code, position = input offset of the failing frame or block, provided =
 * dst_cap, written}; codes HCT_B200_ERR_CORRUPTED, _BUFFER_TOO_SMALL,
 * _CHECKSUM, _UNSUPPORTED.  d_src is read only inside each job's range. */
typedef struct {
    uint64_t src_off, src_len; /* input range in d_src */
    uint64_t dst_off, dst_cap; /* output range in d_dst */
} hct_b200_zstd_job;
int hct_b200_zstd_decompress_jobs(hct_b200_ctx *ctx, const uint8_t *d_src,
                                  const hct_b200_zstd_job *d_jobs, uint32_t n, uint8_t *d_dst,
                                  hct_b200_status *d_status, void *stream);
/* Host buffers: in -> out (capacity out_cap), *written = bytes; one job on
 * the GPU, synchronous. */
int hct_b200_zstd_decompress(hct_b200_ctx *ctx, const uint8_t *in, size_t in_len, uint8_t *out,
                             size_t out_cap, size_t *written, hct_b200_error *err);
/* Sum of the frames' content sizes read from their headers (host only);
 * HCT_B200_ERR_UNSUPPORTED when a frame does not record it,
 * HCT_B200_ERR_CORRUPTED when the headers do not parse. */
int hct_b200_zstd_content_size(const uint8_t *in, size_t in_len, uint64_t *size);

/* ---- HoloTensor (spectral fragments) -----------------------------------
 * HoloTensorReader + HoloTensorDecoder for the spectral encoding
 * (crates/haagenti-hct/src/holotensor.rs).  open parses the 96-byte header
 * (HoloTensorHeader::from_bytes, :571-656: magic "HTNS", version 1, XXH3-64
 * of bytes [0, 88) at 88 when flag 0x0001, encoding / compression / dtype
 * codes, shape), the fragment index (24-byte FragmentIndexEntry, :332-380)
 * and the inline one-fragment form of files with total_fragments == 0
 * (:1978-2003); it uploads every SV03 fragment's f32 values once.
 * decode(k) reads fragments 0..k-1 as HoloTensorReader::read_fragment does
 * (:2039-2098: the entry whose index is i, XXH3 of the stored bytes when flag
 * 0x0002) into a SpectralDecoder (:840-1051: "SV03" raster slices, later
 * fragments over earlier ones, the rest zero) and writes its
 * reconstruction, the orthonormal 2-D DCT-III of the rows x cols view of the
 * shape (HoloTensorDecoder::new, :1732-1759), to d_out (rows x cols of
 * out_dtype).  *quality (may be NULL) receives SpectralDecoder::quality, the
 * fraction of positions the k fragments cover.  k == 0 is
 * HCT_B200_ERR_CORRUPTED ("no fragments loaded").  Fragments whose index
 * entry has flag bit 0 are zstd frames (decoded at open on the GPU, as
 * hct_b200_zstd_decompress_jobs; one that does not decode fails the decode
 * that reads it with HCT_B200_ERR_CORRUPTED).  Not decoded, with
 * HCT_B200_ERR_UNSUPPORTED: the random-projection and low-rank encodings and
 * the legacy V1/V2 spectral fragment layouts.  decode is stream-ordered and
 * synchronises once to read the device flag. */
typedef struct {
    uint8_t encoding;    /* 0 spectral, 1 random projection, 2 low-rank */
    uint8_t compression; /* 0 LZ4, 1 Zstd */
    uint16_t flags;
    uint16_t total_fragments; /* as in the header */
    uint16_t min_fragments;
    uint64_t original_size;
    uint64_t seed;
    uint8_t dtype;
    uint8_t ndim;
    uint16_t inline_format; /* 1: the inline one-fragment form */
    uint32_t reserved;
    uint64_t shape[7];
    float quality_curve[4];
    uint64_t rows, cols; /* the decoder's 2-D view of the shape */
} hct_b200_holo_info;

int hct_b200_holo_open(hct_b200_ctx *ctx, const uint8_t *file, size_t len, hct_b200_holo **out,
                       hct_b200_error *err);
int hct_b200_holo_header(const hct_b200_holo *h, hct_b200_holo_info *out);
/* HoloTensorReader::total_fragments (:2025-2031): 1 for the inline form. */
int hct_b200_holo_total_fragments(const hct_b200_holo *h);
/* QualityCurve::predict(k, total) of the header's curve (:199-220). */
float hct_b200_holo_predict_quality(const hct_b200_holo *h, uint32_t k);
/* How many fragments HoloTensorReader::read_to_quality(target) reads
 * (:2164-2187): the first k whose predicted quality reaches target, else all. */
uint32_t hct_b200_holo_fragments_for_quality(const hct_b200_holo *h, float target);
int hct_b200_holo_decode(hct_b200_holo *h, uint32_t num_fragments, void *d_out, int out_dtype,
                         void *stream, float *quality, hct_b200_error *err);
void hct_b200_holo_close(hct_b200_holo *h);

/* ---- HCT reader ---------------------------------------------------------
 * HctReader::new / HctReaderV2::new (crates/haagenti-hct/src/tensor.rs:417-444,
 * 841-922): parse the header, optional quantization metadata and block index of
 * an HCT file held in host memory, validate the v2 header checksum, and upload
 * the compressed data section to the device (one copy).  With
 * validate_checksums != 0 the per-block XXH3-64 checksums are verified on the
 * host first (HctReaderV2::read_block_validated, tensor.rs:941-975). */
int hct_b200_reader_open(hct_b200_ctx *ctx, const uint8_t *file, size_t file_len,
                         int validate_checksums, hct_b200_reader **out, hct_b200_error *err);
/* Re-upload the compressed data of a file with the same layout into an open
 * reader (stream-ordered H2D copy; pinned host memory makes it asynchronous).
 * The reader orders its device buffer across streams by itself: the copy
 * waits for the last decode that read the buffer, and the next decode on any
 * stream waits for the copy, so uploads may run on a copy stream while other
 * tensors decode. */
int hct_b200_reader_upload(hct_b200_reader *r, const uint8_t *file, size_t file_len, void *stream);
int hct_b200_reader_header(const hct_b200_reader *r, hct_b200_header *out);
uint32_t hct_b200_reader_num_blocks(const hct_b200_reader *r);
/* HctReader::decompress_all (tensor.rs:506-515) on the GPU: all blocks in one
 * launch into d_out (capacity out_cap).  Reference semantics: each block's
 * expected size is block_size except the last (tensor.rs:494-500); a short
 * block is truncated and the rest concatenated.  *written = total bytes. */
int hct_b200_reader_decompress_all(hct_b200_reader *r, uint8_t *d_out, size_t out_cap,
                                   size_t *written, void *stream, hct_b200_error *err);
/* Full decode of the tensor into d_out (rows*cols elements of out_dtype):
 *   spectral (flag HCT_B200_FLAG_SPECTRAL_Q4): LZ4 -> INT4 -> scatter -> IDCT;
 *   plain INT4 (dtype I4 without the flag, examples/safetensors_to_int4_hct.rs):
 *     LZ4 -> dequantize_int4. */
int hct_b200_reader_decode(hct_b200_reader *r, void *d_out, int out_dtype, void *stream,
                           hct_b200_error *err);
/* hct_b200_reader_decode split in two: _async enqueues the whole decode on
 * `stream` without any host synchronisation (per-block statuses and the
 * device error flag are copied to pinned host memory behind the kernels);
 * _wait synchronises on that copy and returns what hct_b200_reader_decode
 * would have returned.  d_out is undefined when _wait reports an error.
 * Asynchronous decodes through one context share its scratch and must be
 * issued on one stream. */
int hct_b200_reader_decode_async(hct_b200_reader *r, void *d_out, int out_dtype, void *stream,
                                 hct_b200_error *err);
int hct_b200_reader_wait(hct_b200_reader *r, hct_b200_error *err);
void hct_b200_reader_close(hct_b200_reader *r);

#ifdef __cplusplus
}
#endif

#endif /* HCT_B200_H */
