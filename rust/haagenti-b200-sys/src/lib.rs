//! Raw bindings of `include/hct_b200.h` (ABI version 2), one declaration per
//! exported symbol, in the header's order.  Device pointers are `*mut c_void`
//! / `*const u8` as in C; `stream` is a `cudaStream_t` passed as `*mut c_void`
//! (null = the legacy default stream).
#![allow(non_camel_case_types)]

use std::os::raw::{c_char, c_int, c_void};

pub const HCT_B200_ABI_VERSION: c_int = 2;

pub const HCT_B200_OK: c_int = 0;
pub const HCT_B200_ERR_UNEXPECTED_EOF: c_int = 1;
pub const HCT_B200_ERR_BUFFER_TOO_SMALL: c_int = 2;
pub const HCT_B200_ERR_ZERO_OFFSET: c_int = 3;
pub const HCT_B200_ERR_OFFSET_BEYOND: c_int = 4;
pub const HCT_B200_ERR_INVALID_ARGUMENT: c_int = 16;
pub const HCT_B200_ERR_CORRUPTED: c_int = 17;
pub const HCT_B200_ERR_CHECKSUM: c_int = 18;
pub const HCT_B200_ERR_UNSUPPORTED: c_int = 19;
pub const HCT_B200_ERR_CUDA: c_int = 20;
pub const HCT_B200_ERR_NO_DEVICE: c_int = 21;
pub const HCT_B200_ERR_TIMEOUT: c_int = 22;
pub const HCT_B200_ERR_OUT_OF_MEMORY: c_int = 23;
pub const HCT_B200_ERR_SIZE_MISMATCH: c_int = 24;

pub const HCT_B200_F32: c_int = 0;
pub const HCT_B200_F16: c_int = 1;
pub const HCT_B200_BF16: c_int = 2;

pub const HCT_B200_FLAG_SPECTRAL_Q4: u16 = 0x0100;
pub const HCT_B200_IDCT_AUTO: c_int = 0;
pub const HCT_B200_IDCT_DENSE: c_int = 1;
pub const HCT_B200_IDCT_SCATTER: c_int = 2;

#[repr(C)]
pub struct hct_b200_ctx {
    _p: [u8; 0],
}
#[repr(C)]
pub struct hct_b200_reader {
    _p: [u8; 0],
}
#[repr(C)]
pub struct hct_b200_v3 {
    _p: [u8; 0],
}
#[repr(C)]
pub struct hct_b200_holo {
    _p: [u8; 0],
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct hct_b200_lz4_block {
    pub src_off: u64,
    pub dst_off: u64,
    pub src_len: u32,
    pub dst_cap: u32,
    pub out_size: u32,
    pub reserved: u32,
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct hct_b200_status {
    pub code: i32,
    pub reserved: i32,
    pub position: u64,
    pub provided: u64,
    pub written: u64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct hct_b200_error {
    pub code: i32,
    pub block: i32,
    pub position: u64,
    pub required: u64,
    pub provided: u64,
    pub message: [c_char; 192],
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct hct_b200_header {
    pub version: u32,
    pub algorithm: u8,
    pub dtype: u8,
    pub flags: u16,
    pub original_size: u64,
    pub compressed_size: u64,
    pub block_size: u32,
    pub num_blocks: u32,
    pub rank: u32,
    pub reserved: u32,
    pub shape: [u64; 4],
    pub quant_meta: [u8; 8],
    pub has_quant_meta: u32,
    pub reserved2: u32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct hct_b200_kernel_stats {
    pub name: [c_char; 32],
    pub launches: u64,
    pub total_ms: f64,
    pub work: f64,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct hct_b200_int4_job {
    pub d_data: *const u8,
    pub data_len: u64,
    pub num_elements: u64,
    pub d_out: *mut c_void,
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct hct_b200_zstd_job {
    pub src_off: u64,
    pub src_len: u64,
    pub dst_off: u64,
    pub dst_cap: u64,
}

#[repr(C)]
#[derive(Default, Clone, Copy, Debug)]
pub struct hct_b200_holo_info {
    pub encoding: u8,
    pub compression: u8,
    pub flags: u16,
    pub total_fragments: u16,
    pub min_fragments: u16,
    pub original_size: u64,
    pub seed: u64,
    pub dtype: u8,
    pub ndim: u8,
    pub inline_format: u16,
    pub reserved: u32,
    pub shape: [u64; 7],
    pub quality_curve: [f32; 4],
    pub rows: u64,
    pub cols: u64,
}

#[link(name = "hct_b200")]
extern "C" {
    // ---- context
    pub fn hct_b200_ctx_create(device: c_int, out: *mut *mut hct_b200_ctx) -> c_int;
    pub fn hct_b200_ctx_destroy(ctx: *mut hct_b200_ctx);
    pub fn hct_b200_ctx_reserve(ctx: *mut hct_b200_ctx, rows: u64, cols: u64) -> c_int;
    pub fn hct_b200_status_string(code: c_int) -> *const c_char;
    pub fn hct_b200_abi_version() -> c_int;
    pub fn hct_b200_ctx_set_idct(ctx: *mut hct_b200_ctx, mode: c_int) -> c_int;
    pub fn hct_b200_ctx_profile(ctx: *mut hct_b200_ctx, enable: c_int) -> c_int;
    pub fn hct_b200_ctx_profile_read(ctx: *mut hct_b200_ctx, out: *mut hct_b200_kernel_stats,
                                     max_entries: c_int, count: *mut c_int) -> c_int;

    // ---- LZ4 (block.rs:261-366, decompress.rs:28-73)
    pub fn hct_b200_lz4_decompress_blocks(d_src: *const u8, d_blocks: *const hct_b200_lz4_block,
                                          num_blocks: u32, d_dst: *mut u8,
                                          d_status: *mut hct_b200_status, max_src_len: u64,
                                          stream: *mut c_void) -> c_int;
    pub fn hct_b200_lz4_decompress_with_size(ctx: *mut hct_b200_ctx, input: *const u8,
                                             in_len: usize, output_size: usize, out: *mut u8,
                                             written: *mut usize, err: *mut hct_b200_error)
                                             -> c_int;
    pub fn hct_b200_lz4_decompress_to(ctx: *mut hct_b200_ctx, input: *const u8, in_len: usize,
                                      out: *mut u8, out_len: usize, written: *mut usize,
                                      err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_lz4_max_compressed_size(n: usize) -> usize;
    pub fn hct_b200_lz4_compress_block(input: *const u8, in_len: usize, out: *mut u8,
                                       out_cap: usize, out_len: *mut usize) -> c_int;
    pub fn hct_b200_lz4_compress_chunks(input: *const u8, in_len: usize, block_size: usize,
                                        out: *mut u8, out_stride: usize, lens: *mut u32) -> c_int;
    pub fn hct_b200_quantize_int4(w: *const f32, n: usize, out: *mut u8) -> c_int;
    pub fn hct_b200_quantize_int4_mp(w: *const f32, n: usize, out: *mut u8) -> c_int;
    pub fn hct_b200_spectral_select(coeffs: *const f32, n: usize, k: usize, bitmap: *mut u8,
                                    values: *mut f32, count: *mut usize) -> c_int;

    // ---- INT4 (quantization.rs:82-131, mixed_precision.rs:489-539)
    pub fn hct_b200_dequantize_int4(d_data: *const u8, data_len: usize, num_elements: usize,
                                    d_out: *mut c_void, out_dtype: c_int, written: *mut usize,
                                    stream: *mut c_void) -> c_int;
    pub fn hct_b200_dequantize_int4_batch(jobs: *const hct_b200_int4_job, num_jobs: u32,
                                          out_dtype: c_int, written: *mut usize,
                                          stream: *mut c_void) -> c_int;
    pub fn hct_b200_dequantize_int4_mp(d_data: *const u8, data_len: usize, num_elements: usize,
                                       d_out: *mut c_void, out_dtype: c_int, written: *mut usize,
                                       stream: *mut c_void) -> c_int;

    // ---- IDCT (dct.rs:311-337) and the spectral payload
    pub fn hct_b200_idct_2d(ctx: *mut hct_b200_ctx, d_in: *const f32, d_out: *mut c_void,
                            out_dtype: c_int, width: usize, height: usize, stream: *mut c_void)
                            -> c_int;
    pub fn hct_b200_spectral_q4_decode(ctx: *mut hct_b200_ctx, d_payload: *const u8,
                                       payload_len: usize, rows: usize, cols: usize,
                                       d_out: *mut c_void, out_dtype: c_int, stream: *mut c_void)
                                       -> c_int;
    pub fn hct_b200_spectral_q4_decode_noalloc(d_payload: *const u8, payload_len: usize,
                                               rows: usize, cols: usize, d_out: *mut c_void,
                                               out_dtype: c_int, stream: *mut c_void) -> c_int;

    // ---- HCT V3 fragments (haagenti-cuda decompress.rs:322-438)
    pub fn hct_b200_v3_open(ctx: *mut hct_b200_ctx, data: *const u8, len: usize, rows: u64,
                            cols: u64, out: *mut *mut hct_b200_v3, err: *mut hct_b200_error)
                            -> c_int;
    pub fn hct_b200_v3_num_fragments(v: *const hct_b200_v3) -> c_int;
    pub fn hct_b200_v3_decode(v: *mut hct_b200_v3, d_out: *mut c_void, out_dtype: c_int,
                              stream: *mut c_void, err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_v3_close(v: *mut hct_b200_v3);
    pub fn hct_b200_hct_v3_decode(ctx: *mut hct_b200_ctx, data: *const u8, len: usize, rows: u64,
                                  cols: u64, d_out: *mut c_void, out_dtype: c_int,
                                  stream: *mut c_void, err: *mut hct_b200_error) -> c_int;

    // ---- Zstandard (zstd::decode_all on the GPU)
    pub fn hct_b200_zstd_decompress_jobs(ctx: *mut hct_b200_ctx, d_src: *const u8,
                                         d_jobs: *const hct_b200_zstd_job, n: u32,
                                         d_dst: *mut u8, d_status: *mut hct_b200_status,
                                         stream: *mut c_void) -> c_int;
    pub fn hct_b200_zstd_decompress(ctx: *mut hct_b200_ctx, input: *const u8, in_len: usize,
                                    out: *mut u8, out_cap: usize, written: *mut usize,
                                    err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_zstd_content_size(input: *const u8, in_len: usize, size: *mut u64) -> c_int;

    // ---- HoloTensor (holotensor.rs)
    pub fn hct_b200_holo_open(ctx: *mut hct_b200_ctx, file: *const u8, len: usize,
                              out: *mut *mut hct_b200_holo, err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_holo_header(h: *const hct_b200_holo, out: *mut hct_b200_holo_info) -> c_int;
    pub fn hct_b200_holo_total_fragments(h: *const hct_b200_holo) -> c_int;
    pub fn hct_b200_holo_predict_quality(h: *const hct_b200_holo, k: u32) -> f32;
    pub fn hct_b200_holo_fragments_for_quality(h: *const hct_b200_holo, target: f32) -> u32;
    pub fn hct_b200_holo_decode(h: *mut hct_b200_holo, num_fragments: u32, d_out: *mut c_void,
                                out_dtype: c_int, stream: *mut c_void, quality: *mut f32,
                                err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_holo_close(h: *mut hct_b200_holo);

    // ---- HCT reader (tensor.rs:408-1021)
    pub fn hct_b200_reader_open(ctx: *mut hct_b200_ctx, file: *const u8, file_len: usize,
                                validate_checksums: c_int, out: *mut *mut hct_b200_reader,
                                err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_reader_upload(r: *mut hct_b200_reader, file: *const u8, file_len: usize,
                                  stream: *mut c_void) -> c_int;
    pub fn hct_b200_reader_header(r: *const hct_b200_reader, out: *mut hct_b200_header) -> c_int;
    pub fn hct_b200_reader_num_blocks(r: *const hct_b200_reader) -> u32;
    pub fn hct_b200_reader_decompress_all(r: *mut hct_b200_reader, d_out: *mut u8,
                                          out_cap: usize, written: *mut usize,
                                          stream: *mut c_void, err: *mut hct_b200_error)
                                          -> c_int;
    pub fn hct_b200_reader_decode(r: *mut hct_b200_reader, d_out: *mut c_void, out_dtype: c_int,
                                  stream: *mut c_void, err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_reader_decode_async(r: *mut hct_b200_reader, d_out: *mut c_void,
                                        out_dtype: c_int, stream: *mut c_void,
                                        err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_reader_wait(r: *mut hct_b200_reader, err: *mut hct_b200_error) -> c_int;
    pub fn hct_b200_reader_close(r: *mut hct_b200_reader);
}
