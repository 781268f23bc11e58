"""The allocation-free attention backward, called through its exported C symbol.

``mt_attention_bwd_noalloc`` serves callers that cannot call cudaMalloc (a
host framework that owns all device memory, code that must not risk the device
synchronisation an allocation can cause, plain C callers).  Its scratch lives
in a fixed device array inside the library, so it must give the same result as
the allocating ``attention_bwd`` binding, call after call, up to the array's
size limit.  Bounded-wait timeouts are read from a status word the caller owns
or, when the caller passes none, through ``mt_attention_noalloc_status``.  This
file sits in ``tests/zz_last`` so that pytest collects it after every other
test.
"""

import ctypes
import math

import pytest
import torch

from meshtrain_b200 import ops

pytestmark = pytest.mark.gpu

# The library's static scratch array, in floats (16 MiB).
SCRATCH_FLOATS = 4 << 20

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


def _lib():
    return ctypes.CDLL(ops.extension()._ext.__file__)


def _entry():
    fn = _lib().mt_attention_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = _ARGTYPES
    return fn


def _library_status() -> int:
    """Reads and clears the library's own status word through its C reader."""
    fn = _lib().mt_attention_noalloc_status
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.c_char_p, ctypes.c_int]
    out = ctypes.c_uint32(0xFFFFFFFF)
    err = ctypes.create_string_buffer(256)
    rc = fn(ctypes.byref(out), err, len(err))
    assert rc == 0, err.value.decode()
    return int(out.value)


def _call(fn, dout, q, k, v, o, lse, dq, dk, dv, causal=True, sizes=None, status=None):
    B, S, Hq, hd = q.shape
    Hk = k.shape[2]
    if sizes is not None:
        B, S, Hq, Hk, hd = sizes
    err = ctypes.create_string_buffer(256)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(dout.data_ptr(), dout.stride(1), q.data_ptr(), q.stride(1), k.data_ptr(), k.stride(1),
            v.data_ptr(), v.stride(1), o.data_ptr(), o.stride(1), lse.data_ptr(),
            dq.data_ptr(), dq.stride(1), dk.data_ptr(), dk.stride(1), dv.data_ptr(), dv.stride(1),
            B, S, Hq, Hk, hd, 1.0 / math.sqrt(hd), int(causal), stream,
            None if status is None else status.data_ptr(), err, len(err))
    return rc, err.value.decode()


def _close(out, ref, tol=3e-2):
    out, ref = out.float(), ref.float()
    scale = ref.abs().max().item() + 1e-6
    assert (out - ref).abs().max().item() <= tol * scale


def _scratch_floats(B, S, Hq, hd):
    acc = B * S * Hq * hd
    return (acc + 63) // 64 * 64 + B * Hq * S


CASES = [
    (2, 256, 4, 2, 64),
    (1, 384, 4, 4, 128),
    (1, 2048, 16, 4, 64),     # sequence length of the 0.48B GPT workload, head dim 64
    (2, 1016, 16, 4, 128),    # needs just under the array's size; S not a multiple of the tile
]


@pytest.mark.parametrize("B,S,Hq,Hk,hd", CASES)
def test_noalloc_matches_allocating_entry_point_twice(B, S, Hq, Hk, hd):
    assert _scratch_floats(B, S, Hq, hd) <= SCRATCH_FLOATS
    ops.set_backend("custom")
    fn = _entry()
    torch.manual_seed(1)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the second call must not see the first call's scratch
        q, k, v = (torch.randn(B, S, h, hd, device="cuda").to(torch.bfloat16) for h in (Hq, Hk, Hk))
        do = torch.randn(B, S, Hq, hd, device="cuda").to(torch.bfloat16)
        o, lse = ops.attention(q, k, v, causal=True)
        ref = ops.attention_bwd(do, q, k, v, o, lse, causal=True)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        rc, msg = _call(fn, do, q, k, v, o, lse, dq, dk, dv, status=status)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert int(status.item()) == 0, "a bounded wait in the allocation-free kernels gave up"
        for got, want in zip((dq, dk, dv), ref):
            _close(got, want)
    assert ops.read_status(torch.cuda.current_device()) == 0


def test_noalloc_library_status_word_when_caller_passes_none():
    ops.set_backend("custom")
    fn = _entry()
    torch.manual_seed(2)
    assert _library_status() == 0
    B, S, Hq, Hk, hd = 1, 512, 8, 2, 128
    for _ in range(2):
        q, k, v = (torch.randn(B, S, h, hd, device="cuda").to(torch.bfloat16) for h in (Hq, Hk, Hk))
        do = torch.randn(B, S, Hq, hd, device="cuda").to(torch.bfloat16)
        o, lse = ops.attention(q, k, v, causal=True)
        ref = ops.attention_bwd(do, q, k, v, o, lse, causal=True)
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        rc, msg = _call(fn, do, q, k, v, o, lse, dq, dk, dv)
        assert rc == 0, msg
        torch.cuda.synchronize()
        assert _library_status() == 0
        for got, want in zip((dq, dk, dv), ref):
            _close(got, want)


def test_noalloc_rejects_problems_beyond_its_scratch():
    fn = _entry()
    q = torch.zeros(1, 128, 1, 64, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(1, 1, 128, device="cuda")
    rc, msg = _call(fn, q, q, q, q, q, lse, q, q, q, sizes=(64, 8192, 32, 8, 128))
    assert rc != 0
    assert "scratch" in msg


def test_noalloc_rejects_null_and_misaligned_pointers_before_launching():
    fn = _entry()
    B, S, H, hd = 1, 128, 1, 64
    q = torch.zeros(B, S, H, hd, device="cuda", dtype=torch.bfloat16)
    lse = torch.zeros(B, H, S, device="cuda")
    buf = torch.zeros(B * S * H * hd + 8, device="cuda", dtype=torch.bfloat16)
    shifted = buf[1:1 + B * S * H * hd].view(B, S, H, hd)  # 2-byte offset: not 16-byte aligned
    rc, msg = _call(fn, q, q, q, q, q, lse, shifted, q, q)
    assert rc != 0 and "dq" in msg and "aligned" in msg
    err = ctypes.create_string_buffer(256)
    rc = fn(None, hd, q.data_ptr(), hd, q.data_ptr(), hd, q.data_ptr(), hd, q.data_ptr(), hd, lse.data_ptr(),
            q.data_ptr(), hd, q.data_ptr(), hd, q.data_ptr(), hd, B, S, H, H, hd, 0.125, 1,
            torch.cuda.current_stream().cuda_stream, None, err, len(err))
    assert rc != 0 and "dout" in err.value.decode() and "NULL" in err.value.decode()
