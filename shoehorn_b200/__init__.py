"""shoehorn_b200 — B200-native quantization hot path of shoehorn.

Python mirror of the reference's row API (src/quant.rs:543-630) over the C ABI
of libshoehorn_cuda.so (include/shoehorn_cuda.h).  Device memory and streams
come from PyTorch; every byte of encoding, decoding and error measurement is
computed by the CUDA kernels in shoehorn_b200/csrc.  There is no CPU fallback:
if the library or a CUDA device is missing, the calls raise.
"""
import ctypes
import enum
import os
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libshoehorn_cuda.so")

SHC_OK = 0
_STATUS = {
    0: "ok", -1: "invalid argument", -2: "CUDA runtime error", -3: "IQ point off the lattice",
    -4: "IQ neighbour search found no finite candidate", -5: "timed out", -6: "out of memory",
    -7: "no usable sm_100 device", -8: "request exceeds the fixed scratch of shc_encode_rows_noalloc",
}

SRC_F32, SRC_F16, SRC_BF16 = 0, 1, 30


class GgmlType(enum.IntEnum):
    """ggml type ids (reference gguf.rs:13-83)."""
    F32 = 0
    F16 = 1
    Q4_0 = 2
    Q4_1 = 3
    Q5_0 = 6
    Q5_1 = 7
    Q8_0 = 8
    Q2_K = 10  # no reference counterpart: ggml's block_q2_K layout
    Q3_K = 11  # no reference counterpart: ggml's block_q3_K layout
    Q4_K = 12
    Q5_K = 13
    Q6_K = 14
    IQ2_XXS = 16
    IQ2_XS = 17
    IQ3_XXS = 18
    IQ4_NL = 20
    IQ3_S = 21
    IQ2_S = 22
    IQ4_XS = 23
    BF16 = 30

    def block_layout(self):
        """(elements per block, bytes per block) — gguf.rs:86-107."""
        return _LAYOUT[self]

    def row_bytes(self, n_per_row):
        """gguf.rs:109-113; raises like the reference's assert on a ragged row."""
        bs, tb = self.block_layout()
        if n_per_row % bs != 0:
            raise ValueError(f"row size {n_per_row} not divisible by block {bs}")
        return n_per_row // bs * tb

    def type_name(self):
        return _NAMES.get(self, self.name)


_LAYOUT = {
    GgmlType.F32: (1, 4), GgmlType.F16: (1, 2), GgmlType.BF16: (1, 2), GgmlType.Q4_0: (32, 18),
    GgmlType.Q4_1: (32, 20), GgmlType.Q5_0: (32, 22), GgmlType.Q5_1: (32, 24), GgmlType.Q8_0: (32, 34),
    GgmlType.Q2_K: (256, 84), GgmlType.Q3_K: (256, 110), GgmlType.Q4_K: (256, 144), GgmlType.Q5_K: (256, 176), GgmlType.Q6_K: (256, 210),
    GgmlType.IQ2_XXS: (256, 66), GgmlType.IQ2_XS: (256, 74), GgmlType.IQ2_S: (256, 82),
    GgmlType.IQ3_XXS: (256, 98), GgmlType.IQ3_S: (256, 110), GgmlType.IQ4_NL: (32, 18),
    GgmlType.IQ4_XS: (256, 136),
}
_NAMES = {GgmlType.Q2_K: "Q2_K", GgmlType.Q3_K: "Q3_K", GgmlType.Q4_K: "Q4_K", GgmlType.Q5_K: "Q5_K",
          GgmlType.Q6_K: "Q6_K"}


class ShoehornError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        super().__init__(f"{what}: {_STATUS.get(status, 'status %d' % status)} ({status})")


_lib = None
_lib_lock = threading.Lock()
_vp, _i64, _u32, _i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint32, ctypes.c_int


def lib():
    """Load libshoehorn_cuda.so (raises if it was not built)."""
    global _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m shoehorn_b200.build` (or __graft_entry__.build())")
        L = ctypes.CDLL(LIB_PATH)
        L.shc_init.argtypes = [_i32, ctypes.POINTER(_vp)]
        L.shc_free.argtypes = [_vp]
        L.shc_status_string.restype = ctypes.c_char_p
        L.shc_status_string.argtypes = [_i32]
        L.shc_row_bytes.restype = _i64
        L.shc_row_bytes.argtypes = [_u32, _i64]
        L.shc_type_supported.argtypes = [_u32]
        L.shc_encode_rows.argtypes = [_vp, _u32, _u32, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _vp]
        L.shc_decode_rows.argtypes = [_vp, _u32, _vp, _i64, _i64, _vp, _vp]
        L.shc_row_errors.argtypes = [_vp, _vp, _i32, _u32, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _vp]
        L.shc_sync.argtypes = [_vp, _vp, _i64]
        L.shc_encode_tensor_host.argtypes = [_vp, _u32, _u32, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64]
        L.shc_row_errors_host.argtypes = [_vp, _vp, _i32, _u32, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i64]
        L.shc_launch_count.restype = _i64
        L.shc_launch_count.argtypes = [_vp]
        L.shc_grid_info.argtypes = [_i32, ctypes.POINTER(ctypes.c_int32), ctypes.POINTER(ctypes.c_int32),
                                    ctypes.POINTER(ctypes.c_int64), _vp, _vp]
        _lib = L
        return L


def _check(rc, what):
    if rc != SHC_OK:
        raise ShoehornError(rc, what)


def row_bytes(ty, ne0):
    return int(lib().shc_row_bytes(int(ty), int(ne0)))


def type_supported(ty):
    return bool(lib().shc_type_supported(int(ty)))


def grid_info(which):
    """Compact IQ lattice map and neighbour lists (host only, no GPU)."""
    L = lib()
    gs, ms, nn = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int64()
    _check(L.shc_grid_info(which, ctypes.byref(gs), ctypes.byref(ms), ctypes.byref(nn), None, None), "grid_info")
    kmap = np.zeros(ms.value, dtype=np.int32)
    nb = np.zeros(nn.value, dtype=np.uint32)
    _check(L.shc_grid_info(which, None, None, None, kmap.ctypes.data, nb.ctypes.data), "grid_info")
    return gs.value, kmap, nb


class Context:
    """A library context bound to one CUDA device (shc_init/shc_free)."""

    def __init__(self, device=0):
        import torch  # device memory and streams are torch's
        self.torch = torch
        self.device = int(device)
        h = ctypes.c_void_p()
        _check(lib().shc_init(self.device, ctypes.byref(h)), "shc_init")
        self.handle = h

    def close(self):
        if getattr(self, "handle", None):
            lib().shc_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---------------- helpers ----------------
    def _stream(self, stream):
        if stream is None:
            stream = self.torch.cuda.current_stream(self.device)
        return ctypes.c_void_p(stream.cuda_stream)

    @staticmethod
    def _src_type(t):
        import torch
        if t.dtype == torch.bfloat16:
            return SRC_BF16
        if t.dtype == torch.float16:
            return SRC_F16
        if t.dtype == torch.float32:
            return SRC_F32
        if t.dtype in (torch.int16, torch.uint16):
            return SRC_BF16  # raw BF16 bit patterns
        raise TypeError(f"unsupported source dtype {t.dtype}")

    def _im(self, im):
        if im is None:
            return None, 0
        if im.dtype != self.torch.float32 or not im.is_contiguous() or not im.is_cuda:
            raise TypeError("imatrix must be a contiguous float32 CUDA tensor")
        return ctypes.c_void_p(im.data_ptr()), im.numel()

    def sync(self, stream=None, timeout_ms=600_000):
        _check(lib().shc_sync(self.handle, self._stream(stream), int(timeout_ms)), "shc_sync")

    def launch_count(self):
        return int(lib().shc_launch_count(self.handle))

    # ---------------- tensor-granular API ----------------
    def encode_rows(self, ty, src, im=None, rows_per_mat=0, row0=0, out=None, stream=None, sync=False):
        """Encode a [n_rows, ne0] CUDA tensor (bf16/f16/f32) row by row into `ty`.

        Bytes equal quant.rs:543 encode_row applied to each row with the
        imatrix slice of imatrix.rs:124 row_slice.  Returns a uint8 CUDA
        tensor [n_rows, row_bytes]."""
        torch = self.torch
        ty = GgmlType(ty)
        if src.dim() != 2 or not src.is_contiguous() or not src.is_cuda:
            raise ValueError("src must be a contiguous 2-D CUDA tensor")
        n_rows, ne0 = src.shape
        rb = ty.row_bytes(ne0)
        if out is None:
            out = torch.empty((n_rows, rb), dtype=torch.uint8, device=src.device)
        imp, iml = self._im(im)
        _check(lib().shc_encode_rows(self.handle, int(ty), self._src_type(src), ctypes.c_void_p(src.data_ptr()),
                                     n_rows, ne0, imp, iml, int(rows_per_mat), int(row0),
                                     ctypes.c_void_p(out.data_ptr()), self._stream(stream)), f"encode_rows {ty.name}")
        if sync:
            self.sync(stream)
        return out

    def decode_rows(self, ty, codes, ne0, out=None, stream=None, sync=False):
        torch = self.torch
        ty = GgmlType(ty)
        n_rows = codes.shape[0] if codes.dim() == 2 else codes.numel() // ty.row_bytes(ne0)
        if out is None:
            out = torch.empty((n_rows, ne0), dtype=torch.float32, device=codes.device)
        _check(lib().shc_decode_rows(self.handle, int(ty), ctypes.c_void_p(codes.data_ptr()), n_rows, ne0,
                                     ctypes.c_void_p(out.data_ptr()), self._stream(stream)), f"decode_rows {ty.name}")
        if sync:
            self.sync(stream)
        return out

    def row_errors(self, types, src, im=None, row_step=1, rows_per_mat=0, row0=0, stream=None, sync=True):
        """Fused encode->decode->weighted SSE per sampled row and candidate.

        Returns a float64 CUDA tensor [len(types), n_sampled]: entry [t, i] is
        quant.rs:618 row_error(types[t], row i*row_step, im)."""
        torch = self.torch
        types = [int(GgmlType(t)) for t in types]
        n_rows, ne0 = src.shape
        n_s = (n_rows + row_step - 1) // row_step
        err = torch.empty((len(types), n_s), dtype=torch.float64, device=src.device)
        tarr = (ctypes.c_uint32 * len(types))(*types)
        imp, iml = self._im(im)
        _check(lib().shc_row_errors(self.handle, tarr, len(types), self._src_type(src), ctypes.c_void_p(src.data_ptr()),
                                    n_rows, ne0, imp, iml, int(rows_per_mat), int(row0), int(row_step),
                                    ctypes.c_void_p(err.data_ptr()), self._stream(stream)), "row_errors")
        if sync:
            self.sync(stream)
        return err

    # ---------------- host-buffer API ----------------
    def encode_tensor_host(self, ty, src, im=None, rows_per_mat=0, row0=0, out=None, timeout_ms=600_000):
        """Encode a host array ([n_rows, ne0] uint16 BF16 bits, float16 or
        float32; numpy or pinned torch CPU tensor) into host bytes."""
        ty = GgmlType(ty)
        ptr, n_rows, ne0, st = _host_view(src)
        rb = ty.row_bytes(ne0)
        if out is None:
            out = np.empty((n_rows, rb), dtype=np.uint8)
        optr = _host_ptr(out)
        imp, iml = (None, 0)
        if im is not None:
            im_np = np.ascontiguousarray(im, dtype=np.float32)
            imp, iml = ctypes.c_void_p(im_np.ctypes.data), im_np.size
        _check(lib().shc_encode_tensor_host(self.handle, int(ty), st, ptr, n_rows, ne0, imp, iml, int(rows_per_mat),
                                            int(row0), optr, int(timeout_ms)), f"encode_tensor_host {ty.name}")
        return out

    def row_errors_host(self, types, src, im=None, row_step=1, rows_per_mat=0, row0=0, timeout_ms=600_000):
        types = [int(GgmlType(t)) for t in types]
        ptr, n_rows, ne0, st = _host_view(src)
        n_s = (n_rows + row_step - 1) // row_step
        err = np.zeros((len(types), n_s), dtype=np.float64)
        tarr = (ctypes.c_uint32 * len(types))(*types)
        imp, iml = (None, 0)
        if im is not None:
            im_np = np.ascontiguousarray(im, dtype=np.float32)
            imp, iml = ctypes.c_void_p(im_np.ctypes.data), im_np.size
        _check(lib().shc_row_errors_host(self.handle, tarr, len(types), st, ptr, n_rows, ne0, imp, iml,
                                         int(rows_per_mat), int(row0), int(row_step),
                                         ctypes.c_void_p(err.ctypes.data), int(timeout_ms)), "row_errors_host")
        return err


def _host_view(src):
    """(pointer, n_rows, ne0, src_type) of a 2-D host array."""
    if isinstance(src, np.ndarray):
        if src.ndim != 2 or not src.flags.c_contiguous:
            raise ValueError("host source must be a C-contiguous 2-D array")
        st = {np.dtype(np.uint16): SRC_BF16, np.dtype(np.float16): SRC_F16, np.dtype(np.float32): SRC_F32}.get(src.dtype)
        if st is None:
            raise TypeError(f"unsupported host dtype {src.dtype}")
        return ctypes.c_void_p(src.ctypes.data), src.shape[0], src.shape[1], st
    # torch CPU tensor (possibly pinned)
    if src.dim() != 2 or not src.is_contiguous() or src.is_cuda:
        raise ValueError("host source must be a contiguous 2-D CPU tensor")
    return ctypes.c_void_p(src.data_ptr()), src.shape[0], src.shape[1], Context._src_type(src)


def _host_ptr(out):
    if isinstance(out, np.ndarray):
        return ctypes.c_void_p(out.ctypes.data)
    return ctypes.c_void_p(out.data_ptr())


_default_ctx = None


def default_context(device=None):
    """Process-wide context on the current CUDA device (like the reference's
    process-wide OnceLock grids)."""
    global _default_ctx
    import torch
    dev = torch.cuda.current_device() if device is None else device
    if _default_ctx is None or _default_ctx.device != dev:
        _default_ctx = Context(dev)
    return _default_ctx


# ---------------- reference row API (quant.rs:543-630) ----------------

def _row_tensor(x):
    import torch
    t = torch.as_tensor(np.ascontiguousarray(x, dtype=np.float32)).reshape(1, -1)
    return t.cuda()


def encode_row(ty, x, im=None):
    """quant.rs:543 encode_row on the GPU: f32 row (+ optional imatrix row
    slice) -> encoded bytes (numpy uint8).  Unknown types raise like the
    reference's panic."""
    ty = GgmlType(ty)
    ctx = default_context()
    xt = _row_tensor(x)
    imt = None if im is None else _row_tensor(im).reshape(-1)
    out = ctx.encode_rows(ty, xt, imt, sync=True)
    return out.cpu().numpy().reshape(-1)


def decode_row(ty, data, n):
    """quant.rs:581 decode_row on the GPU."""
    import torch
    ty = GgmlType(ty)
    ctx = default_context()
    codes = torch.as_tensor(np.ascontiguousarray(data, dtype=np.uint8)).reshape(1, -1).cuda()
    return ctx.decode_rows(ty, codes, n, sync=True).cpu().numpy().reshape(-1)


def row_error(ty, x, im=None):
    """quant.rs:618 row_error on the GPU (fused encode/decode/weighted SSE)."""
    ty = GgmlType(ty)
    ctx = default_context()
    xt = _row_tensor(x)
    imt = None if im is None else _row_tensor(im).reshape(-1)
    return float(ctx.row_errors([ty], xt, imt).cpu()[0, 0])
