"""The allocation-free acceptance entry point, d2sd_verify_accept_noalloc.

It serves callers that cannot allocate device memory when they verify, such as
a serving runtime whose memory planner owns every allocation, or code running
inside a CUDA graph capture. It keeps its scratch in a static device array of
the library instead of a caller-provided workspace. This test calls it through
the C ABI and checks that it returns exactly what d2sd_verify_accept (with a
workspace) returns, on two calls in a row, so the second call also shows that
the shared array is left in a usable state. The file name makes pytest
collect it last.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(gen, B, T, V, dtype, device):
    z = torch.randn(B, T, V, generator=gen).to(dtype)
    x = torch.randint(0, V, (B, T), generator=gen)
    keep = torch.rand(B, T, generator=gen) < 0.8
    x[:, 1:] = torch.where(keep[:, 1:], z.float().argmax(-1)[:, :-1], x[:, 1:])
    return z.to(device), x.to(device)


def _with_workspace(lib, z, x, dtype_code, stream):
    B, T, V = z.shape
    nbytes = lib.d2sd_verify_accept_workspace_size(B, T, V)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=z.device)
    res = torch.zeros(2, dtype=torch.int32, device=z.device)
    acc = torch.zeros(T, dtype=torch.int64, device=z.device)
    am = torch.zeros(B * T, dtype=torch.int64, device=z.device)
    rc = lib.d2sd_verify_accept(z.data_ptr(), dtype_code, B, T, V, z.stride(0), z.stride(1),
                                x.data_ptr(), x.stride(0), x.stride(1), res.data_ptr(),
                                acc.data_ptr(), am.data_ptr(), ws.data_ptr(), nbytes, stream)
    assert rc == 0, lib.d2sd_last_error()
    return res, acc, am


def _no_alloc(lib, z, x, dtype_code, stream):
    B, T, V = z.shape
    res = torch.full((2,), -5, dtype=torch.int32, device=z.device)
    acc = torch.full((T,), -5, dtype=torch.int64, device=z.device)
    am = torch.full((B * T,), -5, dtype=torch.int64, device=z.device)
    rc = lib.d2sd_verify_accept_noalloc(z.data_ptr(), dtype_code, B, T, V, z.stride(0),
                                        z.stride(1), x.data_ptr(), x.stride(0), x.stride(1),
                                        res.data_ptr(), acc.data_ptr(), am.data_ptr(), stream)
    assert rc == 0, lib.d2sd_last_error()
    return res, acc, am


@pytest.mark.parametrize("B,T,V,dtype,code", [
    (8, 32, 151936, torch.bfloat16, 1),   # the north-star verify shape
    (4, 16, 1001, torch.float32, 0),      # odd vocabulary: unaligned rows, scalar path
])
def test_no_alloc_matches_workspace_entry_point(cuda_device, B, T, V, dtype, code):
    from d2sd_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    gen = torch.Generator().manual_seed(B * 1000 + T)
    for call in range(2):  # two calls in a row on the same static scratch
        z, x = _inputs(gen, B, T, V, dtype, cuda_device)
        ra, aa, ma = _with_workspace(lib, z, x, code, stream)
        rb, ab, mb = _no_alloc(lib, z, x, code, stream)
        torch.cuda.synchronize(cuda_device)
        # acceptance is integer work: the bar is bit-exact
        assert torch.equal(ra, rb), (call, ra.tolist(), rb.tolist())
        assert torch.equal(aa, ab), call
        assert torch.equal(ma, mb), call
        acc_len = int(rb[0])
        assert 1 <= acc_len <= T
        assert torch.all(ab[acc_len:] == -1)
        np.testing.assert_array_equal(mb.cpu().numpy(), z.float().argmax(-1).reshape(-1).cpu().numpy())


def test_no_alloc_rejects_oversized_shapes(cuda_device):
    from d2sd_b200 import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    z = torch.zeros(1, dtype=torch.bfloat16, device=cuda_device)
    x = torch.zeros(1, dtype=torch.int64, device=cuda_device)
    r = torch.zeros(2, dtype=torch.int32, device=cuda_device)
    # 64 branches x 1024 positions: more logits rows than the kernel and the
    # static scratch take; rejected before anything is launched
    rc = lib.d2sd_verify_accept_noalloc(z.data_ptr(), 1, 64, 1024, 8, 8, 8, x.data_ptr(), 1, 1,
                                        r.data_ptr(), x.data_ptr(), None, stream)
    assert rc != 0
    assert "scratch" in lib.d2sd_last_error().decode() or "rows" in lib.d2sd_last_error().decode()
