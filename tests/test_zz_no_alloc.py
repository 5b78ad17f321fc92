"""The allocation-free decode-attention entry point, called through its exported C symbol.

For callers that cannot allocate device memory at call time (see the comment block above
``vlmrl_decode_attention_noalloc`` in csrc/attention.cu).  The test compares two consecutive calls
against the regular ``vlmrl.ops.decode_attn`` on the same inputs.  The file is named to be collected
last, so a run that stops at the first failure has already run every other test.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from vlmrl.ops._ext import ext

    lib = ctypes.CDLL(ext().__file__)
    fn = lib.vlmrl_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_void_p] + [ctypes.c_int] * 5 + [ctypes.c_float, ctypes.c_void_p]
    return fn


@pytest.mark.parametrize("B,Hq,Hkv,D,Tmax", [(5, 32, 8, 128, 300), (64, 32, 8, 128, 448), (3, 4, 2, 32, 70)])
def test_noalloc_decode_matches_allocating_path(B, Hq, Hkv, D, Tmax):
    from vlmrl import ops

    fn = _lib()
    g = torch.Generator(device="cuda").manual_seed(B * 7 + D)
    q = torch.randn(B, Hq, D, generator=g, device="cuda").bfloat16()
    kc = torch.randn(B, Hkv, Tmax, D, generator=g, device="cuda").bfloat16()
    vc = torch.randn(B, Hkv, Tmax, D, generator=g, device="cuda").bfloat16()
    lens = torch.randint(1, Tmax + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    scale = 1.0 / math.sqrt(D)
    expected = ops.decode_attn(q, kc, vc, lens, scale=scale)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr(), out.data_ptr(), B, Hq, Hkv, Tmax, D,
                scale, stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        err = (out.float() - expected.float()).abs().max().item()
        assert err <= 2e-2 + 2e-2 * expected.float().abs().max().item(), err
    assert ops.ext().read_and_clear_error(torch.cuda.current_device()) == 0


def test_noalloc_rejects_oversized_problem():
    fn = _lib()
    q = torch.zeros(1, 4, 128, device="cuda", dtype=torch.bfloat16)
    # 4096 sequences x 32 heads x >=2 splits x 130 floats exceeds the 4 MiB scratch array
    rc = fn(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), 4096, 32, 8, 4096, 128, 0.1,
            torch.cuda.current_stream().cuda_stream)
    assert rc == -2
