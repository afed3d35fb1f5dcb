"""The allocation-free decode attention entry point.

`hm_decode_attn_noalloc` exists for callers that must not allocate device memory
while they decode (a real-time audio thread, where cudaMalloc can synchronise the
device and stall, or an application that serves all device memory from its own
fixed arena).  It keeps its scratch in a fixed array inside the library instead of
taking a workspace.  This test calls it through the C ABI twice in a row (the
array keeps the previous call's contents) and checks it against the allocating
entry point, `hm_decode_attn`, and against the oracle's restatement of the
reference kernel, with the tolerance the other attention tests use.
"""
import math

import pytest
import torch

from oracle import heartmula_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def lib():
    from estudiocanciones_b200 import _lib, build
    build.build()
    return _lib.lib()


def _case(seed, R, S, Hq, Hk, hd, L, pos):
    g = torch.Generator().manual_seed(seed)
    B = R // S
    q = torch.randn(R, Hq * hd, generator=g).half().to(DEV)
    kc = torch.randn(B, Hk, L, hd, generator=g).half().to(DEV)
    vc = torch.randn(B, Hk, L, hd, generator=g).half().to(DEV)
    return q, kc, vc, torch.tensor(pos, dtype=torch.long, device=DEV)


def test_noalloc_attention_matches_allocating_entry_point(lib):
    from estudiocanciones_b200 import kernels
    err = kernels.error_word(DEV)
    stream = torch.cuda.current_stream().cuda_stream
    # two calls in a row with different shapes and split counts: the shared scratch
    # array still holds the first call's partials and tickets when the second starts
    cases = [(1, 8, 1, 24, 8, 128, 1350, [975, 0, 1349, 31, 600, 1000, 7, 1200], 10),
             (2, 4, 1, 8, 4, 384, 300, [299, 150, 3, 0], 6)]
    for seed, R, S, Hq, Hk, hd, L, pos, ns in cases:
        q, kc, vc, p = _case(seed, R, S, Hq, Hk, hd, L, pos)
        ref = torch.empty(R, Hq * hd, dtype=torch.float16, device=DEV)
        kernels.attn(q, kc, vc, p, ref, S, Hq, Hk, L, nsplit=ns)
        out = torch.full_like(ref, float("nan"))
        rc = lib.hm_decode_attn_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), p.data_ptr(), out.data_ptr(),
                                        R, S, Hq, Hk, hd, L, 1.0 / math.sqrt(hd), ns, err.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(out.float(), ref.float(), atol=2e-3, rtol=5e-3)
        # and directly against the oracle's restatement of the reference kernel (_attn +
        # _attn_combine, app/kernels.py:112-167) on the host
        orc = O.decode_attn(q.cpu(), kc.cpu(), vc.cpu(), p.cpu(), S, Hq, Hk)
        torch.testing.assert_close(out.float().cpu(), orc.float(), atol=2e-3, rtol=5e-3)
    assert kernels.read_errors(DEV) == 0


def test_noalloc_attention_rejects_requests_beyond_its_scratch(lib):
    from estudiocanciones_b200._lib import HM_ENOSPACE
    q, kc, vc, p = _case(3, 64, 1, 64, 8, 128, 64, [63] * 64)
    out = torch.empty(64, 64 * 128, dtype=torch.float16, device=DEV)
    # 64 rows x 64 heads x 64 splits x 130 floats = 34M floats > the 1M-float array
    rc = lib.hm_decode_attn_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), p.data_ptr(), out.data_ptr(),
                                    64, 1, 64, 8, 128, 64, 0.088, 64, None, torch.cuda.current_stream().cuda_stream)
    assert rc == HM_ENOSPACE
