"""The allocation-free attention backward entry point.

Some callers of this library cannot allocate GPU memory (memory arenas that
own the whole device, host applications that forbid device allocation after
start-up, launch paths that must not reach an allocator).  For them the
library exports ``wb_attn_bwd_noalloc``, a C function whose only scratch
buffer is a fixed-size static device array.  This test calls it through its
exported C symbol (ctypes), on two calls in a row with different inputs, and
checks each result against the regular attention backward entry point, with
the same tolerance as the attention tests.  It also checks that a problem
larger than the static scratch is rejected.  The file name sorts last so a
stop-at-first-failure run has executed every other test before this one.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_ROWS = 1 << 20
ERR_TOO_LARGE = 1


def _lib(cuda_ext):
    lib = ctypes.CDLL(cuda_ext.__file__)
    fn = lib.wb_attn_bwd_noalloc
    i64, i32, vp = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p
    fn.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32,
                   ctypes.c_float, vp]
    fn.restype = i32
    lib.wb_attn_bwd_noalloc_status.argtypes = [i32]
    lib.wb_attn_bwd_noalloc_status.restype = i32
    lib.wb_attn_bwd_noalloc_strerror.argtypes = [i32]
    lib.wb_attn_bwd_noalloc_strerror.restype = ctypes.c_char_p
    return lib


def _problem(seed, lens, hq, hk):
    from wavelet_b200.ops.attention import attention_fwd

    g = torch.Generator(device="cuda").manual_seed(seed)
    T = sum(lens)
    W = (hq + 2 * hk) * 128
    qkv = torch.randn(T, W, device="cuda", dtype=torch.bfloat16, generator=g)
    q = qkv[:, : hq * 128].view(T, hq, 128)
    k = qkv[:, hq * 128 : (hq + hk) * 128].view(T, hk, 128)
    v = qkv[:, (hq + hk) * 128 :].view(T, hk, 128)
    cu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device="cuda")
    out, lse = attention_fwd(q, k, v, cu, max(lens), True)
    do = torch.randn(T, hq, 128, device="cuda", dtype=torch.bfloat16, generator=g)
    return q, k, v, cu, out, lse, do, max(lens)


def _call(lib, q, k, v, cu, out, lse, do, max_len, scale):
    T, hq, _ = q.shape
    hk = k.shape[1]
    dq = torch.empty(T, hq, 128, device="cuda", dtype=torch.bfloat16)
    dk = torch.empty(T, hk, 128, device="cuda", dtype=torch.bfloat16)
    dv = torch.empty(T, hk, 128, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.wb_attn_bwd_noalloc(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                 out.data_ptr(), out.stride(0), lse.data_ptr(), do.data_ptr(), dq.data_ptr(),
                                 dk.data_ptr(), dv.data_ptr(), cu.data_ptr(), cu.numel() - 1, max_len, T, hq, hk,
                                 scale, stream)
    return rc, dq, dk, dv


def test_noalloc_backward_matches_regular_entry_point(cuda_ext):
    from wavelet_b200.ops.attention import attention_bwd

    lib = _lib(cuda_ext)
    scale = 128 ** -0.5
    for seed, lens, hq, hk in ((0, [300, 77, 256], 4, 2), (1, [129, 640, 5], 8, 2)):
        q, k, v, cu, out, lse, do, max_len = _problem(seed, lens, hq, hk)
        want = attention_bwd(do, q, k, v, out, lse, cu, max_len, True, scale)
        rc, dq, dk, dv = _call(lib, q, k, v, cu, out, lse, do, max_len, scale)
        assert rc == 0, lib.wb_attn_bwd_noalloc_strerror(rc)
        torch.cuda.synchronize()
        assert lib.wb_attn_bwd_noalloc_status(torch.cuda.current_device()) == 0
        for got, ref, name in ((dq, want[0], "dq"), (dk, want[1], "dk"), (dv, want[2], "dv")):
            err = (got.float() - ref.float()).abs().max().item()
            tol = 3e-2 * ref.float().abs().max().item() + 3e-2
            assert err <= tol, (seed, name, err, tol)


def test_noalloc_rejects_oversized_problem(cuda_ext):
    lib = _lib(cuda_ext)
    q, k, v, cu, out, lse, do, max_len = _problem(2, [256], 2, 1)
    T_fake = MAX_ROWS // q.shape[1] + 1  # Hq * T just above the static capacity
    dq = torch.empty(1, device="cuda")
    rc = lib.wb_attn_bwd_noalloc(q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0), v.data_ptr(), v.stride(0),
                                 out.data_ptr(), out.stride(0), lse.data_ptr(), do.data_ptr(), dq.data_ptr(),
                                 dq.data_ptr(), dq.data_ptr(), cu.data_ptr(), 1, max_len, T_fake, q.shape[1],
                                 k.shape[1], 1.0, torch.cuda.current_stream().cuda_stream)
    assert rc == ERR_TOO_LARGE
    assert b"capacity" in lib.wb_attn_bwd_noalloc_strerror(rc)
