"""The allocation-free decode-attention entry point, called through its C symbol.

``graspo_paged_decode_attention_noalloc`` (declared in csrc/graspo_noalloc.h)
serves callers that must not allocate device memory when they call the
library: serving processes whose HBM is carved up by their own arena
allocator, C/C++ hosts without a PyTorch allocator to borrow scratch from,
and latency-critical paths that cannot take cudaMalloc's synchronisation.
Its scratch lives in an array compiled into the library.

This test loads the symbol with ctypes, as such a caller would, and checks it
against the regular entry point (which takes a caller-provided scratch
tensor) on two calls in a row -- the second call reuses the array, counters
included, left behind by the first -- for GQA group sizes 1, 4 and 8 and page
sizes 16 and 64, and once against an fp32 PyTorch oracle that shares no code
with either entry point.  The file name sorts last, so a stop-at-first-failure
run has already run every other test.
"""

import ctypes
import math
import re
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

HEADER = Path(__file__).resolve().parents[1] / "csrc" / "graspo_noalloc.h"


def _header_constants() -> dict:
    text = HEADER.read_text()
    consts = {m.group(1): int(m.group(2)) for m in re.finditer(r"(GB_NOALLOC_[A-Z_]+) = (\d+)", text)}
    consts["SCRATCH_FLOATS"] = 1 << int(re.search(r"GRASPO_NOALLOC_SCRATCH_FLOATS \(1L << (\d+)\)", text).group(1))
    return consts


def _symbol():
    import graspo_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    fn = lib.graspo_paged_decode_attention_noalloc
    fn.restype = ctypes.c_int
    # the prototype in csrc/graspo_noalloc.h: 7 pointers, 7 ints, float, int*, stream
    fn.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_int] * 7 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _case(seed: int, G: int, page: int):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows, nkv, D = 6, 4, 128
    nq = nkv * G
    max_pages = max(2, 192 // page)
    pages = rows * max_pages
    kp = torch.randn(pages, nkv, page, D, device="cuda", generator=g).bfloat16()
    vp = torch.randn(pages, nkv, page, D, device="cuda", generator=g).bfloat16()
    q = torch.randn(rows, nq, D, device="cuda", generator=g).bfloat16()
    bt = torch.randperm(pages, device="cuda", generator=g).int().view(rows, max_pages).contiguous()
    cap = max_pages * page
    start = torch.tensor([0, 3, 0, 9, 1, 0], device="cuda", dtype=torch.int32)
    length = torch.tensor([5, 40, 17, cap - 1, 33, cap], device="cuda", dtype=torch.int32)
    return q, kp, vp, bt, start, length, (rows, nq, nkv, page, max_pages, pages)


def _call(fn, q, kp, vp, bt, start, length, out, dims, splits, scale, err):
    rows, nq, nkv, page, max_pages, pages = dims
    stream = torch.cuda.current_stream().cuda_stream
    return fn(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), bt.data_ptr(), start.data_ptr(), length.data_ptr(),
              out.data_ptr(), rows, nq, nkv, page, max_pages, pages, splits, scale, err.data_ptr(), stream)


def _oracle(q, kp, vp, bt, start, length, scale):
    """fp32 attention of each row over its keys [start, len), gathered page by page."""
    rows, nq, D = q.shape
    nkv = kp.shape[1]
    G = nq // nkv
    out = torch.empty(rows, nq, D, device=q.device)
    for r in range(rows):
        keys = torch.cat([kp[int(p)] for p in bt[r]], 1)[:, int(start[r]) : int(length[r])].float()
        vals = torch.cat([vp[int(p)] for p in bt[r]], 1)[:, int(start[r]) : int(length[r])].float()
        qq = q[r].float().view(nkv, G, D)
        out[r] = (torch.softmax(qq @ keys.transpose(1, 2) * scale, -1) @ vals).reshape(nq, D)
    return out.view(rows, nq * D)


@pytest.mark.parametrize("G,page", [(1, 16), (4, 64), (8, 64), (4, 16)])
def test_noalloc_entry_point_matches_regular_entry_point(G, page):
    from graspo_b200.ops._ext import check_errors, ext

    fn = _symbol()
    ok = _header_constants()["GB_NOALLOC_OK"]
    splits = 3
    scale = 1.0 / math.sqrt(128)
    err = torch.zeros(1, device="cuda", dtype=torch.int32)
    for call in range(2):
        q, kp, vp, bt, start, length, dims = _case(seed=call + 10 * G + page, G=G, page=page)
        rows, nq, nkv = dims[:3]
        ref = torch.empty(rows, nq * 128, device="cuda", dtype=torch.bfloat16)
        scratch = torch.zeros(rows * nq * splits * 130 + rows * nkv, device="cuda")
        ext().paged_decode_attention(q, kp, vp, bt, start, length, ref, scale, splits, scratch)
        out = torch.full_like(ref, float("nan"))
        rc = _call(fn, q, kp, vp, bt, start, length, out, dims, splits, scale, err)
        assert rc == ok, f"call {call}: status {rc}"
        torch.cuda.synchronize()
        rel = (out.float() - ref.float()).abs().max().item() / (ref.float().abs().max().item() + 1e-6)
        assert rel < 1e-2, f"call {call}: max rel err {rel}"
        if call == 1 and G == 4 and page == 64:
            want = _oracle(q, kp, vp, bt, start, length, scale)
            rel = (out.float() - want).abs().max().item() / (want.abs().max().item() + 1e-6)
            assert rel < 2e-2, f"fp32 oracle: max rel err {rel}"
    assert int(err.item()) == 0
    check_errors()


def test_noalloc_entry_point_rejects_oversized_and_bad_requests():
    consts = _header_constants()
    fn = _symbol()
    q, kp, vp, bt, start, length, dims = _case(seed=5, G=8, page=16)
    rows, nq, nkv, page, max_pages, pages = dims
    out = torch.zeros(rows, nq * 128, device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, device="cuda", dtype=torch.int32)
    # 4096 rows x 32 heads x 16 splits x 130 floats is far beyond the fixed array
    big_rows = 4096
    assert big_rows * nq * 16 * 130 > consts["SCRATCH_FLOATS"]
    rc = _call(fn, q, kp, vp, bt, start, length, out, (big_rows, nq, nkv, page, max_pages, pages), 16, 0.1, err)
    assert rc == consts["GB_NOALLOC_TOO_LARGE"]
    rc = _call(fn, q, kp, vp, bt, start, length, out, (rows, nq, nkv, page, max_pages, 0), 3, 0.1, err)
    assert rc == consts["GB_NOALLOC_BAD_ARGUMENT"], "num_pages <= 0 must be rejected"
    torch.cuda.synchronize()
    assert int(out.abs().sum().item()) == 0, "a rejected call must launch nothing"
