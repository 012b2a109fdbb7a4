"""shc_encode_rows_noalloc: the encode entry point for callers that cannot
allocate device memory where they encode (a host program whose allocator
already reserved the GPU's memory, or one that must not trigger the
synchronisation cudaMalloc/cudaFree can cause).  Its scratch is a fixed
buffer inside the library, shared by every call and never cleared, so the
test makes two calls in a row with different data and checks both against
shc_encode_rows, byte for byte (the tolerance the parity tests use).

This file is collected last on purpose."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import Q4_K, Q5_K, Q6_K, NAMES, sweep_rows, student_rows

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
import shoehorn_b200 as sh  # noqa: E402

SHC_ETOOLARGE = -8
MAX_ROWS = 65536


def noalloc():
    f = sh.lib().shc_encode_rows_noalloc
    v, i64 = ctypes.c_void_p, ctypes.c_int64
    f.argtypes = [ctypes.c_uint32, ctypes.c_uint32, v, i64, i64, v, i64, i64, i64, v, v]
    f.restype = ctypes.c_int
    return f


@pytest.mark.parametrize("ty", [Q4_K, Q5_K, Q6_K], ids=lambda t: NAMES[t])
def test_noalloc_matches_encode_rows_on_consecutive_calls(ctx, ty):
    f = noalloc()
    stream = torch.cuda.current_stream()
    calls = [sweep_rows(96, 2048, seed=11 + ty), student_rows(40, 4096, seed=12 + ty)]
    for bits, im in calls:
        src = torch.from_numpy(bits.view(np.int16)).cuda()
        imt = torch.from_numpy(im).cuda()
        want = ctx.encode_rows(ty, src, imt, sync=True)
        out = torch.full_like(want, 0xA5)  # caller-owned output, filled with garbage
        rc = f(ty, sh.SRC_BF16, src.data_ptr(), src.shape[0], src.shape[1], imt.data_ptr(), imt.numel(), 0, 0,
               out.data_ptr(), stream.cuda_stream)
        assert rc == 0, sh.lib().shc_status_string(rc)
        torch.cuda.synchronize()
        assert torch.equal(out, want), NAMES[ty]
        # and against the CPU restatement of the reference encoder directly
        assert np.array_equal(out.cpu().numpy(), O.encode_tensor_bf16(ty, bits, im)), NAMES[ty]


def call(f, ty, src, imt, out, rows_per_mat=0, row0=0, n_rows=None):
    stream = torch.cuda.current_stream()
    n = src.shape[0] if n_rows is None else n_rows
    return f(ty, sh.SRC_BF16, src.data_ptr(), n, src.shape[1], None if imt is None else imt.data_ptr(),
             0 if imt is None else imt.numel(), rows_per_mat, row0, out.data_ptr(), stream.cuda_stream)


@pytest.mark.parametrize("ty", [Q4_K, Q6_K], ids=lambda t: NAMES[t])
def test_noalloc_at_its_row_limit(ctx, ty):
    """Exactly SHC_NOALLOC_MAX_ROWS rows fill the fixed buffer: every row
    equals shc_encode_rows, and sampled rows equal the oracle."""
    f = noalloc()
    bits, im = sweep_rows(MAX_ROWS, 256, seed=40 + ty)
    src = torch.from_numpy(bits.view(np.int16)).cuda()
    imt = torch.from_numpy(im).cuda()
    want = ctx.encode_rows(ty, src, imt, sync=True)
    out = torch.full_like(want, 0x5A)
    assert call(f, ty, src, imt, out) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, want), NAMES[ty]
    rows = np.array([0, 1, 4097, 32768, MAX_ROWS - 2, MAX_ROWS - 1])
    assert np.array_equal(out.cpu().numpy()[rows], O.encode_tensor_bf16(ty, bits[rows], im)), NAMES[ty]


@pytest.mark.parametrize("ty", [Q4_K, Q5_K, Q6_K], ids=lambda t: NAMES[t])
def test_noalloc_split_by_row0_with_expert_imatrix(ctx, ty):
    """A tensor of two 48-row matrices with a two-matrix imatrix, encoded as
    two row ranges (row0 = 0 and 40, the second range crossing the matrix
    boundary): the bytes equal one shc_encode_rows call over all rows."""
    f = noalloc()
    bits, _ = sweep_rows(96, 512, seed=60 + ty)
    rng = np.random.default_rng(61 + ty)
    im2 = np.exp(rng.normal(0, 1, 2 * 512)).astype(np.float32)
    src = torch.from_numpy(bits.view(np.int16)).cuda()
    imt = torch.from_numpy(im2).cuda()
    want = ctx.encode_rows(ty, src, imt, rows_per_mat=48, sync=True)
    out = torch.full_like(want, 0xC3)
    assert call(f, ty, src[:40], imt, out[:40], rows_per_mat=48, row0=0) == 0
    assert call(f, ty, src[40:], imt, out[40:], rows_per_mat=48, row0=40) == 0
    torch.cuda.synchronize()
    assert torch.equal(out, want), NAMES[ty]


def test_noalloc_rejects_negative_row_indices(ctx):
    f = noalloc()
    bits, im = sweep_rows(4, 256, seed=3)
    src = torch.from_numpy(bits.view(np.int16)).cuda()
    imt = torch.from_numpy(np.concatenate([im, im])).cuda()
    out = torch.empty((4, 144), dtype=torch.uint8, device="cuda")
    assert call(f, Q4_K, src, imt, out, rows_per_mat=2, row0=-1) == -1
    assert call(f, Q4_K, src, imt, out, rows_per_mat=-2, row0=0) == -1


def test_noalloc_rejects_more_rows_than_its_buffer(ctx):
    f = noalloc()
    rc = f(Q4_K, sh.SRC_BF16, 256, MAX_ROWS + 1, 256, None, 0, 0, 0, 256, None)
    assert rc == SHC_ETOOLARGE
    assert sh.lib().shc_status_string(rc) == b"request exceeds the fixed scratch of shc_encode_rows_noalloc"
