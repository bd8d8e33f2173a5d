"""The allocation-free decode-attention entry point, called through its C symbol.

``graspo_paged_decode_attention_noalloc`` serves callers that must not
allocate device memory (fixed-arena serving processes, C/C++ hosts without a
PyTorch allocator, latency-critical paths that cannot afford cudaMalloc's
synchronisation): its scratch lives in an array compiled into the library.
This test loads the symbol with ctypes, as such a caller would, and checks it
against the regular entry point (which takes a caller-provided scratch
tensor) on two calls in a row -- the second call reuses the array left behind
by the first.  The file name sorts last so a stop-at-first-failure run has
already run every other test.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    import graspo_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.graspo_paged_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_void_p]
    return fn


def _case(seed: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows, nq, nkv, D, page, max_pages = 6, 32, 8, 128, 16, 6
    pages = rows * max_pages
    kp = torch.randn(pages, nkv, page, D, device="cuda", generator=g).bfloat16()
    vp = torch.randn(pages, nkv, page, D, device="cuda", generator=g).bfloat16()
    q = torch.randn(rows, nq, D, device="cuda", generator=g).bfloat16()
    bt = torch.randperm(pages, device="cuda", generator=g).int().view(rows, max_pages).contiguous()
    start = torch.tensor([0, 3, 0, 9, 1, 0], device="cuda", dtype=torch.int32)
    length = torch.tensor([5, 40, 17, 96, 33, 64], device="cuda", dtype=torch.int32)
    return q, kp, vp, bt, start, length, (rows, nq, nkv, page, max_pages)


def test_noalloc_entry_point_matches_regular_entry_point():
    from graspo_b200.ops._ext import check_errors, ext

    fn = _symbol()
    splits = 3
    scale = 1.0 / math.sqrt(128)
    for call in range(2):
        q, kp, vp, bt, start, length, (rows, nq, nkv, page, max_pages) = _case(seed=call)
        ref = torch.empty(rows, nq * 128, device="cuda", dtype=torch.bfloat16)
        scratch = torch.zeros(rows * nq * splits * 130 + rows * nkv, device="cuda")
        ext().paged_decode_attention(q, kp, vp, bt, start, length, ref, scale, splits, scratch)
        out = torch.full_like(ref, float("nan"))
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), start.data_ptr(), length.data_ptr(),
                out.data_ptr(), rows, nq, nkv, page, max_pages, splits, scale, stream)
        assert rc == 0, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs().max().item()
        assert err / (ref.float().abs().max().item() + 1e-6) < 1e-2, f"call {call}: max err {err}"
    check_errors()


def test_noalloc_entry_point_rejects_oversized_requests():
    fn = _symbol()
    q, kp, vp, bt, start, length, (rows, nq, nkv, page, max_pages) = _case(seed=5)
    out = torch.zeros(rows, nq * 128, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    # 4096 rows x 32 heads x 16 splits x 130 floats is far beyond the 4 MiB array
    rc = fn(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), start.data_ptr(), length.data_ptr(),
            out.data_ptr(), 4096, nq, nkv, page, max_pages, 16, 0.1, stream)
    assert rc == 1
    assert int(out.abs().sum().item()) == 0, "a rejected call must launch nothing"
