"""The allocation-free attention-backward entry point, called through its exported C
symbol, against the regular (allocating) entry point.

Callers that cannot call cudaMalloc (engines that reserve all device memory in a fixed
pool at start-up, plain C / FFI hosts without PyTorch's allocator) use
``nori_attention_bwd_noalloc``; it must produce the
same gradients as ``ops.attention_bwd`` on consecutive calls, since every call reuses the
same fixed scratch array. This file is collected last on purpose.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from synthefy_nori_b200 import ops

    ext = ops.lib()
    so = ctypes.CDLL(ext.__file__)
    fn = so.nori_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.POINTER(ctypes.c_int64)] * 7 + [ctypes.c_int64] * 4 + [
        ctypes.c_double, ctypes.c_void_p]
    err = so.nori_attention_bwd_noalloc_error
    err.restype = ctypes.c_char_p
    return fn, err


def _arr(t):
    return (ctypes.c_int64 * 6)(*[int(v) for v in t])


def test_noalloc_attention_bwd_matches_allocating_entry_point():
    from synthefy_nori_b200 import ops

    fn, _ = _lib()
    torch.manual_seed(0)
    BH, Nq, Nk, D = 6, 150, 230, 56
    scale = 1 / math.sqrt(D)
    q = torch.zeros(BH, Nq, 64, device="cuda", dtype=torch.bfloat16)
    k = torch.zeros(BH, Nk, 64, device="cuda", dtype=torch.bfloat16)
    v = torch.zeros(BH, Nk, 64, device="cuda", dtype=torch.bfloat16)
    for t in (q, k, v):
        t[..., :D] = torch.randn(t.shape[0], t.shape[1], D, device="cuda").to(torch.bfloat16)
    hm = lambda n: (n * 64, 0, 0, 64, 1, 1)  # noqa: E731
    tm = lambda n: (n * D, 0, 0, D, 1, 1)  # noqa: E731
    o = torch.empty(BH, Nq, D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(BH, Nq, device="cuda")
    ops.attention_fwd(q, k, v, o, lq=hm(Nq), lk=hm(Nk), lv=hm(Nk), lo=tm(Nq), BH=BH, Nq=Nq, Nk=Nk, d=D, scale=scale,
                      lse=lse)
    do = torch.randn(BH, Nq, D, device="cuda").to(torch.bfloat16)
    # regular entry point
    dq_ref = torch.zeros(BH, Nq, 64, device="cuda")
    dk_ref = torch.empty(BH, Nk, D, device="cuda", dtype=torch.bfloat16)
    dv_ref = torch.empty(BH, Nk, D, device="cuda", dtype=torch.bfloat16)
    ops.attention_bwd(q, k, v, o, do, lse, dq_ref, dk_ref, dv_ref, lq=hm(Nq), lk=hm(Nk), lv=hm(Nk), lo=tm(Nq),
                      ldo=tm(Nq), ldk=tm(Nk), ldv=tm(Nk), BH=BH, Nq=Nq, Nk=Nk, d=D, scale=scale)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # two calls in a row share (and must reset) the scratch
        dq = torch.full((BH, Nq, 64), 7.0, device="cuda")  # not zeroed: the entry point clears it
        dk = torch.empty(BH, Nk, D, device="cuda", dtype=torch.bfloat16)
        dv = torch.empty(BH, Nk, D, device="cuda", dtype=torch.bfloat16)
        rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(), dq.data_ptr(),
                dk.data_ptr(), dv.data_ptr(), _arr(hm(Nq)), _arr(hm(Nk)), _arr(hm(Nk)), _arr(tm(Nq)), _arr(tm(Nq)),
                _arr(tm(Nk)), _arr(tm(Nk)), BH, Nq, Nk, D, scale, stream)
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(dq, dq_ref, atol=1e-4, rtol=1e-4)
        torch.testing.assert_close(dk.float(), dk_ref.float(), atol=1e-2, rtol=1e-2)
        torch.testing.assert_close(dv.float(), dv_ref.float(), atol=1e-2, rtol=1e-2)


def test_noalloc_rejects_oversized_problem():
    fn, err = _lib()
    z = torch.zeros(16, device="cuda")
    lay = _arr((0, 0, 0, 64, 1, 1))
    rc = fn(*([z.data_ptr()] * 9), lay, lay, lay, lay, lay, lay, lay, 2048, 1024, 64, 64, 0.125, 0)
    assert rc != 0
    assert b"NORI_NOALLOC_MAX_ROWS" in err()


def _valid_args(n=16):
    z = torch.zeros(4096, device="cuda")
    lay = (0, 0, 0, 64, 1, 1)
    return z, lay


def test_noalloc_rejects_misaligned_pointer_without_side_effects():
    fn, err = _lib()
    z, lay = _valid_args()
    dq = torch.full((64,), 3.0, device="cuda")
    ptrs = [z.data_ptr()] * 9
    ptrs[0] = z.data_ptr() + 2  # q misaligned
    ptrs[6] = dq.data_ptr()
    a = _arr(lay)
    rc = fn(*ptrs, a, a, a, a, a, a, a, 1, 1, 1, 64, 0.125, 0)
    torch.cuda.synchronize()
    assert rc != 0 and b"aligned" in err()
    assert bool((dq == 3.0).all())  # nothing was queued: dq not cleared


def test_noalloc_rejects_zero_layout_divisor():
    fn, err = _lib()
    z, _ = _valid_args()
    dq = torch.full((64,), 3.0, device="cuda")
    ptrs = [z.data_ptr()] * 9
    ptrs[6] = dq.data_ptr()
    good, bad = _arr((0, 0, 0, 64, 1, 1)), _arr((0, 0, 0, 64, 1, 0))  # d2 = 0
    rc = fn(*ptrs, good, bad, good, good, good, good, good, 1, 1, 1, 64, 0.125, 0)
    torch.cuda.synchronize()
    assert rc != 0 and b"d1 and d2" in err()
    assert bool((dq == 3.0).all())
    # a stride that is not a multiple of 8 elements is rejected too
    odd = _arr((0, 0, 0, 60, 1, 1))
    rc = fn(*ptrs, odd, good, good, good, good, good, good, 1, 1, 1, 64, 0.125, 0)
    assert rc != 0 and b"multiples of 8" in err()
