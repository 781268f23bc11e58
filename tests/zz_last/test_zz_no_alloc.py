"""The allocation-free attention backward, called through its exported C symbol.

``mt_attention_bwd_noalloc`` serves callers that cannot call cudaMalloc (a
host framework that owns all device memory, code that must not risk the device
synchronisation an allocation can cause, plain C callers).  Its scratch lives
in a fixed device array inside the library, so it must give the same result as
the allocating ``attention_bwd`` binding, call after call.  This file sits in
``tests/zz_last`` so that pytest collects it after every other test.
"""

import ctypes
import math

import pytest
import torch

from meshtrain_b200 import ops

pytestmark = pytest.mark.gpu

_ARGTYPES = [
    ctypes.c_void_p, ctypes.c_long,  # dout, ld_do
    ctypes.c_void_p, ctypes.c_long,  # q
    ctypes.c_void_p, ctypes.c_long,  # k
    ctypes.c_void_p, ctypes.c_long,  # v
    ctypes.c_void_p, ctypes.c_long,  # o
    ctypes.c_void_p,                 # lse
    ctypes.c_void_p, ctypes.c_long,  # dq
    ctypes.c_void_p, ctypes.c_long,  # dk
    ctypes.c_void_p, ctypes.c_long,  # dv
    ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,  # B, S, Hq, Hk, hd
    ctypes.c_float, ctypes.c_int,    # scale, causal
    ctypes.c_void_p,                 # stream
    ctypes.c_void_p,                 # device status word (NULL: the library's own)
    ctypes.c_char_p, ctypes.c_int,   # err, errlen
]


def _entry():
    path = ops.extension()._ext.__file__
    fn = ctypes.CDLL(path).mt_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = _ARGTYPES
    return fn


def _call(fn, dout, q, k, v, o, lse, dq, dk, dv, causal=True, sizes=None):
    B, S, Hq, hd = q.shape
    Hk = k.shape[2]
    if sizes is not None:
        B, S, Hq, Hk, hd = sizes
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(dout.data_ptr(), dout.stride(1), q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1),
            v.data_ptr(), v.stride(1), o.data_ptr(), o.stride(1), lse.data_ptr(),
            dq.data_ptr(), dq.stride(1), dk.data_ptr(), dk.stride(1), dv.data_ptr(), dv.stride(1),
            B, S, Hq, Hk, hd, 1.0 / math.sqrt(hd), int(causal), stream, None, err, len(err))
    return rc, err.value.decode()


def _close(out, ref, tol=3e-2):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    assert (out - ref).abs().max().item() <= tol * scale


@pytest.mark.parametrize("B,S,Hq,Hk,hd", [(2, 256, 4, 2, 64), (1, 384, 4, 4, 128)])
def test_noalloc_matches_allocating_entry_point_twice(B, S, Hq, Hk, hd):
    ops.set_backend("custom")
    fn = _entry()
    torch.manual_seed(1)
    for _ in range(2):  # the second call must not see the first call's scratch
        q, k, v = (torch.randn(B, S, h, hd, device="cuda").to(torch.bfloat16) for h in (Hq, Hk, Hk))
        do = torch.randn(B, S, Hq, hd, device="cuda").to(torch.bfloat16)
        o, lse = ops.attention(q, k, v, causal=True)
        ref = ops.attention_bwd(do, q, k, v, o, lse, causal=True)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        rc, msg = _call(fn, do, q, k, v, o, lse, dq, dk, dv)
        assert rc == 0, msg
        torch.cuda.synchronize()
        for got, want in zip((dq, dk, dv), ref):
            _close(got, want)
    assert ops.read_status(torch.cuda.current_device()) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    fn = _entry()
    q = torch.zeros(1, 128, 1, 64, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(1, 1, 128, device="cuda")
    rc, msg = _call(fn, q, q, q, q, q, lse, q, q, q, sizes=(64, 8192, 32, 8, 128))
    assert rc != 0
    assert "scratch" in msg
