"""haagenti_b200: B200-native HCT weight decode behind the reference's API.

Python mirror of the reference's interfaces for this path, calling the
CUDA library (libhct_b200.so) through its C ABI:

* ``Lz4Decompressor`` -- haagenti_lz4::Lz4Decompressor's ``Decompressor``
  surface (crates/haagenti-lz4/src/decompress.rs:28-73), decoded on the GPU,
  plus a batched ``decompress_blocks`` for many independent blocks.
* ``dequantize_int4`` -- haagenti::testing::dequantize_int4
  (crates/haagenti/src/testing/quantization.rs:82-131); ``dequantize_int4_mp``
  -- the mixed-precision pair's zero-filling form (crates/haagenti/src/
  mixed_precision.rs:489-539).
* ``idct_2d`` -- haagenti_core::dct::idct_2d (crates/haagenti-core/src/dct.rs:311-337).
* ``HctReader`` / ``HctReaderV2`` -- crates/haagenti-hct/src/tensor.rs:408-516,
  832-1021, with ``decompress_all`` on the GPU and ``decode`` for the full
  LZ4 -> INT4 -> IDCT pipeline.

Errors are raised as ``HaagentiError`` subclasses named after the
haagenti_core::Error variants (crates/haagenti-core/src/error.rs:10-65).
Device buffers are torch CUDA tensors (plumbing only).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from ._lib import BF16, F16, F32, FLAG_SPECTRAL_Q4

IDCT_AUTO, IDCT_DENSE, IDCT_SCATTER = 0, 1, 2

__all__ = [
    "HaagentiError", "CorruptedData", "BufferTooSmall", "UnexpectedEof", "ChecksumMismatch",
    "Unsupported", "DeviceError", "Context", "Lz4Decompressor", "dequantize_int4",
    "dequantize_int4_mp", "idct_2d",
    "spectral_q4_decode", "HctReader", "HctReaderV2", "HctV3Decoder", "hct_v3_decode",
    "HoloTensorReader", "ZstdDecompressor", "ZstdGpuPipeline", "zstd_decompress", "F32",
    "F16", "BF16", "FLAG_SPECTRAL_Q4",
]


class HaagentiError(Exception):
    def __init__(self, code: int, message: str, block: int = -1, position: int = 0,
                 required: int = 0, provided: int = 0):
        super().__init__(message)
        self.code, self.block, self.position = code, block, position
        self.required, self.provided = required, provided


class CorruptedData(HaagentiError):
    pass


class BufferTooSmall(HaagentiError):
    pass


class UnexpectedEof(HaagentiError):
    @property
    def bytes_read(self) -> int:
        return self.position


class ChecksumMismatch(CorruptedData):
    pass


class Unsupported(HaagentiError):
    pass


class DeviceError(HaagentiError):
    pass


_CLASS = {
    L.UNEXPECTED_EOF: UnexpectedEof, L.BUFFER_TOO_SMALL: BufferTooSmall,
    L.ZERO_OFFSET: CorruptedData, L.OFFSET_BEYOND: CorruptedData, L.CORRUPTED: CorruptedData,
    L.CHECKSUM: ChecksumMismatch, L.UNSUPPORTED: Unsupported, L.SIZE_MISMATCH: CorruptedData,
}


def _raise(code: int, err: L.Error | None = None):
    lib = L.load()
    if err is not None and err.code:
        msg = err.message.decode(errors="replace") or lib.hct_b200_status_string(code).decode()
        cls = _CLASS.get(code, DeviceError)
        raise cls(code, msg, err.block, err.position, err.required, err.provided)
    raise _CLASS.get(code, DeviceError)(code, lib.hct_b200_status_string(code).decode())


def _check(code: int, err: L.Error | None = None):
    if code != L.OK:
        _raise(code, err)


def _torch():
    import torch

    return torch


def _stream_ptr(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


_DT = {F32: "float32", F16: "float16", BF16: "bfloat16"}


def _torch_dtype(dt: int):
    return getattr(_torch(), _DT[dt])


def _as_host_u8(data) -> np.ndarray:
    if isinstance(data, np.ndarray):
        return np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    return np.frombuffer(bytes(data), dtype=np.uint8)


class Context:
    """One per device: scratch memory, cached DCT bases (GpuContext's role)."""

    _default: dict = {}

    def __init__(self, device: int = 0):
        lib = L.load()
        h = C.c_void_p()
        _check(lib.hct_b200_ctx_create(device, C.byref(h)))
        self._h = h
        self.device = device

    @classmethod
    def default(cls, device: int | None = None) -> "Context":
        if device is None:
            device = _torch().cuda.current_device()
        if device not in cls._default:
            cls._default[device] = Context(device)
        return cls._default[device]

    @property
    def handle(self):
        return self._h

    def reserve(self, rows: int, cols: int):
        _check(L.load().hct_b200_ctx_reserve(self._h, rows, cols))

    def set_idct(self, mode: int):
        """IDCT_AUTO (factored tcgen05 DFT stages when the lengths factor) or IDCT_DENSE."""
        _check(L.load().hct_b200_ctx_set_idct(self._h, mode))

    def close(self):
        if getattr(self, "_h", None):
            L.load().hct_b200_ctx_destroy(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover - interpreter teardown order
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ LZ4

class Lz4Decompressor:
    """GPU implementation of the reference's ``Decompressor`` trait for LZ4."""

    def __init__(self, ctx: Context | None = None):
        self.ctx = ctx or Context.default()

    @staticmethod
    def algorithm() -> str:
        return "lz4"

    def _call(self, data, cap: int, output_size: int) -> bytes:
        lib = L.load()
        src = _as_host_u8(data)
        out = np.zeros(max(cap, 1), dtype=np.uint8)
        written = C.c_size_t(0)
        err = L.Error()
        if cap == output_size:
            fn = lib.hct_b200_lz4_decompress_with_size
            rc = fn(self.ctx.handle, src.ctypes.data if src.size else None, src.size, output_size,
                    out.ctypes.data, C.byref(written), C.byref(err))
        else:
            raise ValueError("capacity must equal output size")
        _check(rc, err)
        return out[: written.value].tobytes()

    def decompress_with_size(self, data, output_size: int) -> bytes:
        """decompress.rs:63-68: block decode into output_size bytes, truncated to the result."""
        return self._call(data, output_size, output_size)

    def decompress_to(self, data, output) -> int:
        """decompress.rs:59-61: decode into ``output`` (a writable buffer); returns bytes written."""
        mv = memoryview(output).cast("B")
        res = self._call(data, len(mv), len(mv))
        mv[: len(res)] = res
        return len(res)

    def decompress(self, data) -> bytes:
        """decompress.rs:33-57: unknown size; start at 4x input, double on BufferTooSmall."""
        src = _as_host_u8(data)
        size = src.size * 4
        while True:
            try:
                return self.decompress_with_size(src, size)
            except BufferTooSmall as e:
                size = max(e.required, size * 2)
                if size > 256 * 1024 * 1024:
                    raise CorruptedData(L.CORRUPTED, "corrupted data: decompressed size exceeds limit")

    def decompress_blocks(self, d_src, blocks: np.ndarray, d_dst, stream=None, staged=True):
        """Batched block decode on device buffers.

        ``blocks`` is a structured array of (src_off, dst_off, src_len, dst_cap,
        out_size) rows; returns the per-block status array (code, position,
        provided, written), synchronising the stream.  The largest src_len is
        passed as the kernel's size bound (``staged=False`` passes none, which
        selects the variant that parses straight from device memory).
        """
        torch = _torch()
        blk = np.zeros(len(blocks), dtype=[("src_off", "<u8"), ("dst_off", "<u8"),
                                           ("src_len", "<u4"), ("dst_cap", "<u4"),
                                           ("out_size", "<u4"), ("reserved", "<u4")])
        for f in ("src_off", "dst_off", "src_len", "dst_cap", "out_size"):
            blk[f] = blocks[f]
        dev = d_src.device
        d_blk = torch.from_numpy(blk.view(np.uint8).copy()).to(dev)
        d_st = torch.zeros(len(blocks) * 32, dtype=torch.uint8, device=dev)
        bound = int(blk["src_len"].max()) if staged and len(blk) else 0
        _check(L.load().hct_b200_lz4_decompress_blocks(
            d_src.data_ptr(), d_blk.data_ptr(), len(blocks), d_dst.data_ptr(), d_st.data_ptr(),
            bound, _stream_ptr(stream)))
        st = d_st.cpu().numpy().view([("code", "<i4"), ("reserved", "<i4"), ("position", "<u8"),
                                       ("provided", "<u8"), ("written", "<u8")])
        return st


# ------------------------------------------------------------------ INT4

def dequantize_int4(data, num_elements: int, out_dtype: int = F32, device=None, stream=None):
    """quantization.rs:82-131 on the GPU; returns a CUDA tensor of ``written`` elements.

    ``data`` is a CUDA uint8 tensor or host bytes (copied to the device first).
    """
    torch = _torch()
    if not (hasattr(data, "is_cuda") and data.is_cuda):
        host = _as_host_u8(data)
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        data = torch.from_numpy(host.copy()).to(dev)
    out = torch.empty(max(num_elements, 1), dtype=_torch_dtype(out_dtype), device=data.device)
    written = C.c_size_t(0)
    _check(L.load().hct_b200_dequantize_int4(data.data_ptr(), data.numel(), num_elements,
                                             out.data_ptr(), out_dtype, C.byref(written),
                                             _stream_ptr(stream)))
    return out[: written.value]


def dequantize_int4_batch(items, out_dtype: int = F32, outs=None, stream=None):
    """Many dequantize_int4 calls in few launches: ``items`` is a list of
    (CUDA uint8 tensor, num_elements); returns one CUDA tensor of ``written``
    elements per item (into ``outs`` when given)."""
    torch = _torch()
    n = len(items)
    jobs = (L.Int4Job * max(n, 1))()
    res = []
    for i, (data, num) in enumerate(items):
        out = (outs[i] if outs is not None else
               torch.empty(max(num, 1), dtype=_torch_dtype(out_dtype), device=data.device))
        jobs[i] = L.Int4Job(data.data_ptr(), data.numel(), num, out.data_ptr())
        res.append(out)
    written = (C.c_size_t * max(n, 1))()
    _check(L.load().hct_b200_dequantize_int4_batch(jobs, n, out_dtype, written,
                                                   _stream_ptr(stream)))
    return [r[: written[i]] for i, r in enumerate(res)]


def dequantize_int4_mp(data, num_elements: int, out_dtype: int = F32, device=None, stream=None):
    """mixed_precision.rs:489-539 on the GPU: ``num_elements`` values, zero where
    the data runs short (an empty tensor for ``num_elements == 0`` or empty data)."""
    torch = _torch()
    if not (hasattr(data, "is_cuda") and data.is_cuda):
        host = _as_host_u8(data)
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        data = torch.from_numpy(host.copy()).to(dev)
    out = torch.empty(max(num_elements, 1), dtype=_torch_dtype(out_dtype), device=data.device)
    written = C.c_size_t(0)
    _check(L.load().hct_b200_dequantize_int4_mp(data.data_ptr(), data.numel(), num_elements,
                                                out.data_ptr(), out_dtype, C.byref(written),
                                                _stream_ptr(stream)))
    return out[: written.value]


# ------------------------------------------------------------------ IDCT

def idct_2d(coeffs, width: int | None = None, height: int | None = None, out_dtype: int = F32,
            ctx: Context | None = None, stream=None):
    """dct.rs:311 idct_2d of a (height, width) f32 CUDA tensor on tcgen05 tensor cores."""
    torch = _torch()
    x = coeffs.contiguous().to(torch.float32)
    if height is None or width is None:
        height, width = (1, x.numel()) if x.dim() == 1 else (x.shape[-2], x.shape[-1])
    ctx = ctx or Context.default(x.device.index)
    out = torch.empty((height, width), dtype=_torch_dtype(out_dtype), device=x.device)
    _check(L.load().hct_b200_idct_2d(ctx.handle, x.data_ptr(), out.data_ptr(), out_dtype, width,
                                     height, _stream_ptr(stream)))
    return out


def spectral_q4_decode(payload, rows: int, cols: int, out_dtype: int = F32,
                       ctx: Context | None = None, stream=None):
    """Decode a device-resident spectral payload (bitmap ++ INT4) to a rows x cols tensor."""
    torch = _torch()
    ctx = ctx or Context.default(payload.device.index)
    out = torch.empty((rows, cols), dtype=_torch_dtype(out_dtype), device=payload.device)
    _check(L.load().hct_b200_spectral_q4_decode(ctx.handle, payload.data_ptr(), payload.numel(),
                                                rows, cols, out.data_ptr(), out_dtype,
                                                _stream_ptr(stream)))
    return out


# ------------------------------------------------------------------ HCT V3 fragments

class HctV3Decoder:
    """GpuDecompressor::decompress for HCT V3 fragment data
    (crates/haagenti-cuda/src/decompress.rs:322-438; ref/c/hct_decoder.h:322-394):
    bitmap + fp16 coefficients per fragment, scattered and inverse-DCT'd on the GPU."""

    def __init__(self, data, rows: int, cols: int, ctx: Context | None = None):
        self.ctx = ctx or Context.default()
        self._data = _as_host_u8(data)
        self.rows, self.cols = int(rows), int(cols)
        h = C.c_void_p()
        err = L.Error()
        _check(L.load().hct_b200_v3_open(self.ctx.handle,
                                         self._data.ctypes.data if self._data.size else None,
                                         self._data.size, self.rows, self.cols, C.byref(h),
                                         C.byref(err)), err)
        self._h = h

    @property
    def num_fragments(self) -> int:
        return int(L.load().hct_b200_v3_num_fragments(self._h))

    def decode(self, out_dtype: int = F32, out=None, stream=None):
        torch = _torch()
        if out is None:
            out = torch.empty((self.rows, self.cols), dtype=_torch_dtype(out_dtype),
                              device=torch.device("cuda", self.ctx.device))
        err = L.Error()
        _check(L.load().hct_b200_v3_decode(self._h, out.data_ptr(), out_dtype, _stream_ptr(stream),
                                           C.byref(err)), err)
        return out

    def close(self):
        if getattr(self, "_h", None):
            L.load().hct_b200_v3_close(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def hct_v3_decode(data, rows: int, cols: int, out_dtype: int = F32, ctx: Context | None = None,
                  stream=None):
    """One-shot form (the reference C decoder's hct_decode(data, len, rows, cols))."""
    d = HctV3Decoder(data, rows, cols, ctx)
    try:
        return d.decode(out_dtype, stream=stream)
    finally:
        d.close()


# ------------------------------------------------------------------ Zstandard

class ZstdDecompressor:
    """GPU Zstandard decode with the semantics of ``zstd::decode_all``, which the
    reference calls for zstd-compressed HoloTensor fragments
    (crates/haagenti-hct/src/holotensor.rs:2081-2091) and zstd-wrapped HCT data
    (crates/haagenti-cuda/src/decompress.rs:296-319)."""

    def __init__(self, ctx: Context | None = None):
        self.ctx = ctx or Context.default()

    @staticmethod
    def algorithm() -> str:
        return "zstd"

    @staticmethod
    def content_size(data) -> int | None:
        """Sum of the frames' recorded content sizes, None if a frame lacks one."""
        src = _as_host_u8(data)
        size = C.c_uint64(0)
        rc = L.load().hct_b200_zstd_content_size(src.ctypes.data if src.size else None, src.size,
                                                 C.byref(size))
        if rc == L.UNSUPPORTED:
            return None
        _check(rc)
        return int(size.value)

    def decompress_with_size(self, data, capacity: int) -> bytes:
        """Decode every frame into at most ``capacity`` bytes (BufferTooSmall beyond)."""
        src = _as_host_u8(data)
        out = np.zeros(max(capacity, 1), dtype=np.uint8)
        written = C.c_size_t(0)
        err = L.Error()
        _check(L.load().hct_b200_zstd_decompress(self.ctx.handle,
                                                 src.ctypes.data if src.size else None, src.size,
                                                 out.ctypes.data, capacity, C.byref(written),
                                                 C.byref(err)), err)
        return out[: written.value].tobytes()

    def decompress(self, data) -> bytes:
        """decode_all: the recorded content size, else 4x the input doubled on
        BufferTooSmall."""
        src = _as_host_u8(data)
        known = self.content_size(src) if src.size else 0
        size = known if known is not None else max(4 * src.size, 4096)
        while True:
            try:
                return self.decompress_with_size(src, size)
            except BufferTooSmall:
                if known is not None or size >= 1 << 32:
                    raise
                size *= 2

    def decompress_jobs(self, d_src, jobs: np.ndarray, d_dst, stream=None):
        """Batched decode on device buffers: ``jobs`` is a structured array of
        (src_off, src_len, dst_off, dst_cap) rows; returns the per-job status
        array (code, position, provided, written), synchronising the stream."""
        torch = _torch()
        jobs = np.ascontiguousarray(jobs)
        n = len(jobs)
        dev = torch.device("cuda", self.ctx.device)
        d_jobs = torch.from_numpy(jobs.view(np.uint8).copy()).to(dev)
        d_status = torch.zeros(max(n, 1) * 32, dtype=torch.uint8, device=dev)
        _check(L.load().hct_b200_zstd_decompress_jobs(self.ctx.handle, d_src.data_ptr(),
                                                      d_jobs.data_ptr(), n, d_dst.data_ptr(),
                                                      d_status.data_ptr(), _stream_ptr(stream)))
        st = d_status.cpu().numpy()[: n * 32].view(
            [("code", "<i4"), ("reserved", "<i4"), ("position", "<u8"), ("provided", "<u8"),
             ("written", "<u8")])
        return st


def zstd_decompress(data, ctx: Context | None = None) -> bytes:
    """``zstd::decode_all(data)`` on the GPU."""
    return ZstdDecompressor(ctx).decompress(data)


class ZstdGpuPipeline:
    """The reference's GPU zstd pipeline interface
    (crates/haagenti-cuda/src/zstd_gpu.rs:348-402: is_ready, decompress,
    decompress_with_dict, decompress_batch, decompress_to_gpu), decoding on the
    GPU: a batch in one launch, ``decompress_to_gpu`` without a host round trip
    of the output.  Dictionaries are not supported (Unsupported)."""

    def __init__(self, ctx: Context | None = None):
        self.z = ZstdDecompressor(ctx)

    @staticmethod
    def is_ready() -> bool:
        return True

    def decompress(self, compressed) -> bytes:
        return self.z.decompress(compressed)

    def decompress_with_dict(self, compressed, dictionary) -> bytes:
        raise Unsupported(L.UNSUPPORTED, "zstd: dictionaries are not supported by the GPU decoder")

    def _device_jobs(self, frames, sizes, stream=None):
        torch = _torch()
        dev = torch.device("cuda", self.z.ctx.device)
        jobs = np.zeros(len(frames), dtype=ZSTD_JOB)
        so = do = 0
        for i, (f, n) in enumerate(zip(frames, sizes)):
            jobs[i] = (so, len(f), do, n)
            so += (len(f) + 15) // 16 * 16
            do += (n + 15) // 16 * 16
        src = np.zeros(max(so, 16), np.uint8)
        for i, f in enumerate(frames):
            src[int(jobs[i]["src_off"]): int(jobs[i]["src_off"]) + len(f)] = np.frombuffer(f, np.uint8)
        d_dst = torch.empty(max(do, 16), dtype=torch.uint8, device=dev)
        st = self.z.decompress_jobs(torch.from_numpy(src).to(dev), jobs, d_dst, stream)
        return jobs, st, d_dst

    def decompress_batch(self, frames) -> list:
        """Every frame of the list in one launch (frames without a recorded
        content size are decoded one by one with growing capacities)."""
        frames = [bytes(f) for f in frames]
        sizes = [self.z.content_size(f) if f else 0 for f in frames]
        known = [i for i, n in enumerate(sizes) if n is not None]
        out: list = [None] * len(frames)
        if known:
            jobs, st, d_dst = self._device_jobs([frames[i] for i in known],
                                                [sizes[i] for i in known])
            host = d_dst.cpu().numpy()
            for k, i in enumerate(known):
                _check(int(st[k]["code"]))
                o = int(jobs[k]["dst_off"])
                out[i] = host[o: o + int(st[k]["written"])].tobytes()
        for i, n in enumerate(sizes):
            if n is None:
                out[i] = self.z.decompress(frames[i])
        return out

    def decompress_to_gpu(self, compressed, stream=None):
        """The decoded bytes as a uint8 tensor on the context's device."""
        f = bytes(compressed)
        known = self.z.content_size(f) if f else 0
        size = known if known is not None else max(4 * len(f), 4096)
        while True:
            jobs, st, d_dst = self._device_jobs([f], [size], stream)
            code = int(st[0]["code"])
            if code == L.BUFFER_TOO_SMALL and known is None and size < 1 << 32:
                size *= 2
                continue
            _check(code)
            return d_dst[: int(st[0]["written"])]


ZSTD_JOB = np.dtype([("src_off", "<u8"), ("src_len", "<u8"), ("dst_off", "<u8"),
                     ("dst_cap", "<u8")])


# ------------------------------------------------------------------ HoloTensor

class HoloTensorReader:
    """HoloTensorReader + HoloTensorDecoder for spectral HoloTensor files
    (crates/haagenti-hct/src/holotensor.rs:1935-2192, 1719-1810) held in
    memory: the header and fragment index parsed on the host, the SV03
    fragments' values uploaded once, and each decode (scatter of the first k
    fragments + 2-D DCT-III) run on the GPU."""

    def __init__(self, file, ctx: Context | None = None):
        self.ctx = ctx or Context.default()
        self._data = _as_host_u8(file)
        h = C.c_void_p()
        err = L.Error()
        _check(L.load().hct_b200_holo_open(self.ctx.handle,
                                           self._data.ctypes.data if self._data.size else None,
                                           self._data.size, C.byref(h), C.byref(err)), err)
        self._h = h
        info = L.HoloInfo()
        _check(L.load().hct_b200_holo_header(self._h, C.byref(info)))
        self.info = info
        self.shape = tuple(int(info.shape[i]) for i in range(info.ndim))
        self.rows, self.cols = int(info.rows), int(info.cols)
        self.quality = None  # SpectralDecoder::quality of the last decode

    @property
    def total_fragments(self) -> int:
        """HoloTensorReader::total_fragments (holotensor.rs:2025-2031)."""
        return int(L.load().hct_b200_holo_total_fragments(self._h))

    @property
    def is_inline_format(self) -> bool:
        return bool(self.info.inline_format)

    def predict_quality(self, k: int) -> float:
        """QualityCurve::predict(k, total) of the header's curve."""
        return float(L.load().hct_b200_holo_predict_quality(self._h, int(k)))

    def fragments_for_quality(self, target: float) -> int:
        """The number of fragments read_to_quality(target) reads."""
        return int(L.load().hct_b200_holo_fragments_for_quality(self._h, float(target)))

    def decode(self, num_fragments: int | None = None, out_dtype: int = F32, out=None,
               stream=None):
        """Reconstruction from fragments 0..k-1 (all by default) as a
        rows x cols tensor; self.quality is the decoder's coverage."""
        torch = _torch()
        k = self.total_fragments if num_fragments is None else int(num_fragments)
        if out is None:
            out = torch.empty((self.rows, self.cols), dtype=_torch_dtype(out_dtype),
                              device=torch.device("cuda", self.ctx.device))
        q = C.c_float(0.0)
        err = L.Error()
        _check(L.load().hct_b200_holo_decode(self._h, k, out.data_ptr(), out_dtype,
                                             _stream_ptr(stream), C.byref(q), C.byref(err)), err)
        self.quality = float(q.value)
        return out

    def decode_to_quality(self, target: float, out_dtype: int = F32, stream=None):
        """decode_from_file_progressive (holotensor.rs:2332-2348): the
        fragments read_to_quality(target) reads, and its predicted quality."""
        k = self.fragments_for_quality(target)
        out = self.decode(k, out_dtype, stream=stream)
        q = 1.0 if self.is_inline_format else self.predict_quality(k)
        return out, q

    def close(self):
        if getattr(self, "_h", None):
            L.load().hct_b200_holo_close(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------ HCT reader

class HctReader:
    """tensor.rs:408-516 over an HCT file held in memory (bytes / numpy)."""

    _validate = False

    def __init__(self, file, ctx: Context | None = None):
        self.ctx = ctx or Context.default()
        self._file = _as_host_u8(file)
        h = C.c_void_p()
        err = L.Error()
        rc = L.load().hct_b200_reader_open(self.ctx.handle, self._file.ctypes.data,
                                           self._file.size, 1 if self._validate else 0,
                                           C.byref(h), C.byref(err))
        _check(rc, err)
        self._h = h
        hdr = L.Header()
        _check(L.load().hct_b200_reader_header(self._h, C.byref(hdr)))
        self._hdr = hdr

    def header(self) -> dict:
        h = self._hdr
        return dict(version=h.version, algorithm=h.algorithm, dtype=h.dtype, flags=h.flags,
                    original_size=h.original_size, compressed_size=h.compressed_size,
                    block_size=h.block_size, num_blocks=h.num_blocks,
                    shape=[int(h.shape[i]) for i in range(min(h.rank, 4))])

    def num_blocks(self) -> int:
        return int(L.load().hct_b200_reader_num_blocks(self._h))

    @property
    def shape(self):
        return self.header()["shape"]

    def upload(self, file, stream=None):
        """Re-upload the compressed data of a same-layout file (stream-ordered).

        The copy may run on its own stream: it waits for the previous decode
        of this reader to finish reading the buffer, and the next decode waits
        for the copy, with no host synchronisation."""
        f = _as_host_u8(file) if not isinstance(file, np.ndarray) else file
        _check(L.load().hct_b200_reader_upload(self._h, f.ctypes.data, f.size, _stream_ptr(stream)))

    def decompress_all(self, stream=None):
        """tensor.rs:506-515 on the GPU: the concatenated payload as a CUDA uint8 tensor."""
        torch = _torch()
        n = self._hdr.original_size
        out = torch.empty(max(n, 1), dtype=torch.uint8,
                          device=torch.device("cuda", self.ctx.device))
        written = C.c_size_t(0)
        err = L.Error()
        rc = L.load().hct_b200_reader_decompress_all(self._h, out.data_ptr(), out.numel(),
                                                     C.byref(written), _stream_ptr(stream),
                                                     C.byref(err))
        _check(rc, err)
        return out[: written.value]

    def decode(self, out_dtype: int = BF16, out=None, stream=None):
        """Full decode (LZ4 -> INT4 -> [scatter -> IDCT]) into a CUDA tensor of the tensor's shape."""
        torch = _torch()
        shape = self.shape
        if out is None:
            out = torch.empty(shape, dtype=_torch_dtype(out_dtype),
                              device=torch.device("cuda", self.ctx.device))
        err = L.Error()
        rc = L.load().hct_b200_reader_decode(self._h, out.data_ptr(), out_dtype,
                                             _stream_ptr(stream), C.byref(err))
        _check(rc, err)
        return out

    def decode_async(self, out, out_dtype: int = BF16, stream=None):
        """Enqueue the full decode into ``out`` with no host sync; call ``wait()`` for the status."""
        err = L.Error()
        rc = L.load().hct_b200_reader_decode_async(self._h, out.data_ptr(), out_dtype,
                                                   _stream_ptr(stream), C.byref(err))
        _check(rc, err)
        return out

    def wait(self):
        """Status of the last ``decode_async`` (raises like ``decode``)."""
        err = L.Error()
        _check(L.load().hct_b200_reader_wait(self._h, C.byref(err)), err)

    def close(self):
        if getattr(self, "_h", None):
            L.load().hct_b200_reader_close(self._h)
            self._h = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


class HctReaderV2(HctReader):
    """tensor.rs:832-1021: v1/v2 files, header checksum, per-block XXH3 validation."""

    _validate = True

    def decompress_all_validated(self, stream=None):
        return self.decompress_all(stream)
