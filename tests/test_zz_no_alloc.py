"""The allocation-free attention backward (C symbol ``kore_attn_bwd_noalloc``).

It exists for callers that cannot allocate GPU memory while they run (their
own memory pool owns the device, allocation is forbidden after start-up, or
they are plain C programs without PyTorch's allocator). This test calls it
through its exported C symbol, twice in a row with different inputs, and
compares each result with the regular entry point that takes caller-provided
scratch. This file is named to be collected last.
"""
import ctypes
import glob
import os

import pytest
import torch

from kore_b200.ops import attention as attn

pytestmark = pytest.mark.gpu

_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib():
    import kore_b200._C  # noqa: F401  (loads the library and its CUDA module)
    path = glob.glob(os.path.join(_ROOT, "kore_b200", "_C*.so"))[0]
    lib = ctypes.CDLL(path)
    fn = lib.kore_attn_bwd_noalloc
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    fn.argtypes = [P, I64, P, I64, P, I64, P, I64, P, P, P, I, I, I, I, I, ctypes.c_float,
                   P, I64, P, I64, P, I64, P]
    fn.restype = ctypes.c_int
    return fn


def _case(lens, hq, hkv, seed):
    torch.manual_seed(seed)
    T, D = sum(lens), 128
    qk = torch.randn(T, (hq + hkv) * D, device="cuda").bfloat16()
    v = torch.randn(T, hkv * D, device="cuda").bfloat16().view(T, hkv, D)
    q = qk[:, : hq * D].view(T, hq, D)
    k = qk[:, hq * D:].view(T, hkv, D)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    o, lse = attn.attn_fwd(q, k, v, cu, max(lens))
    do = torch.randn_like(o)
    return q, k, v, o, lse, do, cu, max(lens)


def _rel(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


def test_noalloc_matches_regular_entry_point_twice():
    fn = _lib()
    for seed, (lens, hq, hkv) in enumerate([([300, 77], 4, 2), ([640], 5, 1)]):
        q, k, v, o, lse, do, cu, mx = _case(lens, hq, hkv, seed)
        dq_ref, dk_ref, dv_ref = attn.attn_bwd(do, q, k, v, o, lse, cu, mx)
        T = q.shape[0]
        dq = torch.full_like(q, float("nan"))
        dk = torch.full(k.shape, float("nan"), dtype=k.dtype, device="cuda")
        dv = torch.full(v.shape, float("nan"), dtype=v.dtype, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        rc = fn(do.data_ptr(), do.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
                v.data_ptr(), v.stride(0), o.data_ptr(), lse.data_ptr(), cu.data_ptr(),
                cu.numel() - 1, mx, T, hq, hkv, 1.0 / 128 ** 0.5, dq.data_ptr(), dq.stride(0),
                dk.data_ptr(), dk.stride(0), dv.data_ptr(), dv.stride(0), stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert _rel(dq, dq_ref) < 2e-2
        assert _rel(dk, dk_ref) < 2e-2
        assert _rel(dv, dv_ref) < 2e-2


def test_noalloc_rejects_oversized_call():
    fn = _lib()
    q, k, v, o, lse, do, cu, mx = _case([256], 2, 1, 3)
    # claim a token count whose scratch would exceed the fixed 64 MiB array
    rc = fn(do.data_ptr(), do.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
            v.data_ptr(), v.stride(0), o.data_ptr(), lse.data_ptr(), cu.data_ptr(), 1, mx,
            1 << 20, 2, 1, 0.088, q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
            v.data_ptr(), v.stride(0), torch.cuda.current_stream().cuda_stream)
    assert rc == 1


def test_noalloc_strided_outputs_and_argument_checks():
    """dq/dk/dv as row-strided views of wider buffers: the gaps between rows
    stay untouched; a row stride that is not a multiple of 8, or narrower than
    a row, is rejected with code 2; the error reader reports a clean run."""
    fn = _lib()
    import kore_b200._C  # noqa: F401
    lib = ctypes.CDLL(glob.glob(os.path.join(_ROOT, "kore_b200", "_C*.so"))[0])
    read_err = lib.kore_attn_noalloc_read_error
    read_err.restype = ctypes.c_int
    lens, hq, hkv = [200, 56], 4, 2
    q, k, v, o, lse, do, cu, mx = _case(lens, hq, hkv, 7)
    dq_ref, dk_ref, dv_ref = attn.attn_bwd(do, q, k, v, o, lse, cu, mx)
    T, D = q.shape[0], 128
    pad = 24
    bq = torch.full((T, hq * D + pad), 7.0, device="cuda").bfloat16()
    bk = torch.full((T, hkv * D + pad), 7.0, device="cuda").bfloat16()
    bv = torch.full((T, hkv * D + pad), 7.0, device="cuda").bfloat16()
    dq, dk, dv = bq[:, : hq * D], bk[:, : hkv * D], bv[:, : hkv * D]
    stream = torch.cuda.current_stream().cuda_stream

    def call(ld_dq, ld_dk):
        return fn(do.data_ptr(), do.stride(0), q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
                  v.data_ptr(), v.stride(0), o.data_ptr(), lse.data_ptr(), cu.data_ptr(), cu.numel() - 1, mx,
                  T, hq, hkv, 1.0 / 128 ** 0.5, dq.data_ptr(), ld_dq, dk.data_ptr(), ld_dk,
                  dv.data_ptr(), bv.stride(0), stream)

    assert call(bq.stride(0), bk.stride(0)) == 0
    torch.cuda.synchronize()
    assert read_err() == 0
    assert _rel(dq.reshape(T, hq, D), dq_ref) < 2e-2
    assert _rel(dk.reshape(T, hkv, D), dk_ref) < 2e-2
    assert _rel(dv.reshape(T, hkv, D), dv_ref) < 2e-2
    for b, w in ((bq, hq * D), (bk, hkv * D), (bv, hkv * D)):
        assert torch.all(b[:, w:] == 7.0)
    assert call(bq.stride(0) - 4, bk.stride(0)) == 2          # not a multiple of 8
    assert call(hq * D - 8, bk.stride(0)) == 2                  # narrower than a row
