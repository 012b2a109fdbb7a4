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


def test_noalloc_rejects_more_rows_than_its_buffer(ctx):
    f = noalloc()
    rc = f(Q4_K, sh.SRC_BF16, 256, MAX_ROWS + 1, 256, None, 0, 0, 0, 256, None)
    assert rc == SHC_ETOOLARGE
    assert sh.lib().shc_status_string(rc) == b"request exceeds the fixed scratch of shc_encode_rows_noalloc"
