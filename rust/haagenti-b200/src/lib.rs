//! Safe layer over `haagenti-b200-sys`: the reference's decode-path interfaces
//! backed by the B200 library.
//!
//! * [`GpuLz4Decompressor`] implements `haagenti_core::Decompressor` with the
//!   semantics of `haagenti_lz4::Lz4Decompressor`
//!   (crates/haagenti-lz4/src/decompress.rs:28-73): the same bytes, the same
//!   error variant and position (block.rs:261-366).
//! * [`ZstdGpu`] implements it for Zstandard frames (`zstd::decode_all`).
//! * [`dequantize_int4`] / [`dequantize_int4_batch`] are
//!   `haagenti::testing::dequantize_int4` (quantization.rs:82-131) on device
//!   buffers.
//! * [`GpuHctReader`] is `HctReader{,V2}` (crates/haagenti-hct/src/tensor.rs:
//!   408-1021) with the whole tensor decoded on the GPU: `decompress_all`
//!   into device memory, or the full decode (LZ4 -> INT4 -> bitmap scatter
//!   -> IDCT) straight to f32/f16/bf16 weights.
//!
//! Device pointers and streams are raw (`*mut c_void`), as the library's C
//! ABI takes them; ownership of device memory stays with the caller.
use haagenti_b200_sys as ffi;
use haagenti_core::{Algorithm, Decompressor, Error, Result};
use std::os::raw::c_void;
use std::sync::Mutex;

fn zero_err() -> ffi::hct_b200_error {
    // SAFETY: a plain C struct of integers and a char array; all-zero is valid
    unsafe { std::mem::zeroed() }
}

/// Library status -> haagenti_core::Error, variant for variant.
pub fn to_error(code: i32, e: &ffi::hct_b200_error) -> Error {
    match code {
        ffi::HCT_B200_ERR_UNEXPECTED_EOF => Error::unexpected_eof(e.position as usize),
        ffi::HCT_B200_ERR_BUFFER_TOO_SMALL => {
            Error::buffer_too_small(e.required as usize, e.provided as usize)
        }
        ffi::HCT_B200_ERR_ZERO_OFFSET => Error::corrupted("invalid zero offset"),
        ffi::HCT_B200_ERR_OFFSET_BEYOND => {
            Error::corrupted_at("offset beyond output", e.position as usize)
        }
        _ => {
            // SAFETY: the library NUL-terminates message; status_string is static
            let msg = unsafe {
                if e.message[0] != 0 {
                    std::ffi::CStr::from_ptr(e.message.as_ptr()).to_string_lossy().into_owned()
                } else {
                    std::ffi::CStr::from_ptr(ffi::hct_b200_status_string(code))
                        .to_string_lossy()
                        .into_owned()
                }
            };
            Error::corrupted(msg)
        }
    }
}

fn check(code: i32, e: &ffi::hct_b200_error) -> Result<()> {
    if code == ffi::HCT_B200_OK {
        Ok(())
    } else {
        Err(to_error(code, e))
    }
}

/// One library context per device (scratch, cached DCT tables).  Calls on a
/// context are serialised by its mutex, as the reference's GpuContext
/// expects of its users (crates/haagenti-cuda/src/lib.rs:99-108).
pub struct Context {
    raw: Mutex<*mut ffi::hct_b200_ctx>,
}
// SAFETY: the raw handle is only used under the mutex
unsafe impl Send for Context {}
unsafe impl Sync for Context {}

impl Context {
    pub fn new(device: i32) -> Result<Self> {
        let mut ctx = std::ptr::null_mut();
        let rc = unsafe { ffi::hct_b200_ctx_create(device, &mut ctx) };
        check(rc, &zero_err())?;
        Ok(Self { raw: Mutex::new(ctx) })
    }
    fn with<T>(&self, f: impl FnOnce(*mut ffi::hct_b200_ctx) -> T) -> T {
        let g = self.raw.lock().unwrap();
        f(*g)
    }
}

impl Drop for Context {
    fn drop(&mut self) {
        let g = self.raw.lock().unwrap();
        unsafe { ffi::hct_b200_ctx_destroy(*g) };
    }
}

/// GPU LZ4 block decoder with the semantics of haagenti_lz4::Lz4Decompressor.
pub struct GpuLz4Decompressor {
    ctx: Context,
}

impl GpuLz4Decompressor {
    pub fn new(device: i32) -> Result<Self> {
        Ok(Self { ctx: Context::new(device)? })
    }
}

impl Decompressor for GpuLz4Decompressor {
    fn algorithm(&self) -> Algorithm {
        Algorithm::Lz4
    }

    fn decompress_to(&self, input: &[u8], output: &mut [u8]) -> Result<usize> {
        let mut written = 0usize;
        let mut err = zero_err();
        let rc = self.ctx.with(|c| unsafe {
            ffi::hct_b200_lz4_decompress_to(c, input.as_ptr(), input.len(), output.as_mut_ptr(),
                                            output.len(), &mut written, &mut err)
        });
        check(rc, &err).map(|_| written)
    }

    fn decompress_with_size(&self, input: &[u8], output_size: usize) -> Result<Vec<u8>> {
        let mut out = vec![0u8; output_size];
        let mut written = 0usize;
        let mut err = zero_err();
        let rc = self.ctx.with(|c| unsafe {
            ffi::hct_b200_lz4_decompress_with_size(c, input.as_ptr(), input.len(), output_size,
                                                   out.as_mut_ptr(), &mut written, &mut err)
        });
        check(rc, &err)?;
        out.truncate(written);
        Ok(out)
    }

    fn decompress(&self, input: &[u8]) -> Result<Vec<u8>> {
        // decompress.rs:33-57: a 4x guess, doubled on BufferTooSmall up to 256 MiB
        let mut size = input.len() * 4;
        loop {
            match self.decompress_with_size(input, size) {
                Err(Error::BufferTooSmall { required, .. }) => {
                    size = required.max(size * 2);
                    if size > 256 * 1024 * 1024 {
                        return Err(Error::corrupted("decompressed size exceeds limit"));
                    }
                }
                r => return r,
            }
        }
    }
}

/// zstd::decode_all on the GPU (RFC 8878 frames; libzstd's bytes).
pub struct ZstdGpu {
    ctx: Context,
}

impl ZstdGpu {
    pub fn new(device: i32) -> Result<Self> {
        Ok(Self { ctx: Context::new(device)? })
    }
}

impl Decompressor for ZstdGpu {
    fn algorithm(&self) -> Algorithm {
        Algorithm::Zstd
    }

    fn decompress_to(&self, input: &[u8], output: &mut [u8]) -> Result<usize> {
        let mut written = 0usize;
        let mut err = zero_err();
        let rc = self.ctx.with(|c| unsafe {
            ffi::hct_b200_zstd_decompress(c, input.as_ptr(), input.len(), output.as_mut_ptr(),
                                          output.len(), &mut written, &mut err)
        });
        check(rc, &err).map(|_| written)
    }

    fn decompress_with_size(&self, input: &[u8], size: usize) -> Result<Vec<u8>> {
        let mut out = vec![0u8; size];
        let n = self.decompress_to(input, &mut out)?;
        out.truncate(n);
        Ok(out)
    }

    fn decompress(&self, input: &[u8]) -> Result<Vec<u8>> {
        // the recorded content size, else growing capacities
        let mut size = 0u64;
        let known = unsafe { ffi::hct_b200_zstd_content_size(input.as_ptr(), input.len(), &mut size) }
            == ffi::HCT_B200_OK;
        let mut cap = if known { size as usize } else { (4 * input.len()).max(4096) };
        loop {
            match self.decompress_with_size(input, cap) {
                Err(Error::BufferTooSmall { .. }) if !known && cap < (1usize << 32) => cap *= 2,
                r => return r,
            }
        }
    }
}

/// quantization.rs:82-131 on device buffers; returns the element count the
/// reference's short-input rules give (known without a device sync).
///
/// # Safety
/// `d_data` must hold `data_len` bytes and `d_out` room for `num_elements`
/// values of `out_dtype` on the current device; `stream` a valid stream or null.
pub unsafe fn dequantize_int4(d_data: *const u8, data_len: usize, num_elements: usize,
                              d_out: *mut c_void, out_dtype: i32, stream: *mut c_void)
                              -> Result<usize> {
    let mut written = 0usize;
    let rc = ffi::hct_b200_dequantize_int4(d_data, data_len, num_elements, d_out, out_dtype,
                                           &mut written, stream);
    check(rc, &zero_err()).map(|_| written)
}

/// Many dequantize_int4 calls in few launches; element counts per job.
///
/// # Safety
/// Every job's buffers as for [`dequantize_int4`].
pub unsafe fn dequantize_int4_batch(jobs: &[ffi::hct_b200_int4_job], out_dtype: i32,
                                    stream: *mut c_void) -> Result<Vec<usize>> {
    let mut written = vec![0usize; jobs.len()];
    let rc = ffi::hct_b200_dequantize_int4_batch(jobs.as_ptr(), jobs.len() as u32, out_dtype,
                                                 written.as_mut_ptr(), stream);
    check(rc, &zero_err()).map(|_| written)
}

/// An HCT file (v1 or v2) opened on the GPU: header, index and checksums
/// parsed on the host, the compressed data uploaded once.
pub struct GpuHctReader<'c> {
    raw: *mut ffi::hct_b200_reader,
    _ctx: &'c Context,
}

impl<'c> GpuHctReader<'c> {
    /// HctReader::new / HctReaderV2::new over the file's bytes; with
    /// `validate_checksums` the per-block XXH3-64 sums are checked first.
    pub fn open(ctx: &'c Context, file: &[u8], validate_checksums: bool) -> Result<Self> {
        let mut raw = std::ptr::null_mut();
        let mut err = zero_err();
        let rc = ctx.with(|c| unsafe {
            ffi::hct_b200_reader_open(c, file.as_ptr(), file.len(), validate_checksums as i32,
                                      &mut raw, &mut err)
        });
        check(rc, &err)?;
        Ok(Self { raw, _ctx: ctx })
    }

    pub fn header(&self) -> ffi::hct_b200_header {
        let mut h = ffi::hct_b200_header::default();
        unsafe { ffi::hct_b200_reader_header(self.raw, &mut h) };
        h
    }

    pub fn num_blocks(&self) -> u32 {
        unsafe { ffi::hct_b200_reader_num_blocks(self.raw) }
    }

    /// HctReader::decompress_all into device memory: all blocks in one launch.
    ///
    /// # Safety
    /// `d_out` must hold `cap` bytes on the reader's device.
    pub unsafe fn decompress_all(&mut self, d_out: *mut u8, cap: usize, stream: *mut c_void)
                                 -> Result<usize> {
        let mut written = 0usize;
        let mut err = zero_err();
        let rc = ffi::hct_b200_reader_decompress_all(self.raw, d_out, cap, &mut written, stream,
                                                     &mut err);
        check(rc, &err).map(|_| written)
    }

    /// The whole decode (spectral: LZ4 -> INT4 -> scatter -> IDCT; plain INT4:
    /// LZ4 -> dequantize_int4) into `d_out` as `out_dtype`.
    ///
    /// # Safety
    /// `d_out` must hold the tensor's elements of `out_dtype`.
    pub unsafe fn decode(&mut self, d_out: *mut c_void, out_dtype: i32, stream: *mut c_void)
                         -> Result<()> {
        let mut err = zero_err();
        let rc = ffi::hct_b200_reader_decode(self.raw, d_out, out_dtype, stream, &mut err);
        check(rc, &err)
    }

    /// `decode` split in two: enqueue without a host sync, then `wait`.
    ///
    /// # Safety
    /// As for [`GpuHctReader::decode`]; `d_out` must stay valid until `wait`.
    pub unsafe fn decode_async(&mut self, d_out: *mut c_void, out_dtype: i32,
                               stream: *mut c_void) -> Result<()> {
        let mut err = zero_err();
        let rc = ffi::hct_b200_reader_decode_async(self.raw, d_out, out_dtype, stream, &mut err);
        check(rc, &err)
    }

    pub fn wait(&mut self) -> Result<()> {
        let mut err = zero_err();
        let rc = unsafe { ffi::hct_b200_reader_wait(self.raw, &mut err) };
        check(rc, &err)
    }
}

impl Drop for GpuHctReader<'_> {
    fn drop(&mut self) {
        unsafe { ffi::hct_b200_reader_close(self.raw) };
    }
}
