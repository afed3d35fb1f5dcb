"""hm_q8_rows (the converter's per-row int8 quantisation on the GPU) bit-identical to
the reference converter's outputs and to the oracle; the GPU converter equal to the
CPU-oracle conversion.  Every call goes through the C ABI."""
import numpy as np
import pytest
import torch

from oracle import heartmula_oracle as O
from estudiocanciones_b200 import _lib, convert

from test_convert_cpu import fake_official, golden_cases

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _built():
    from estudiocanciones_b200 import build
    build.build()


def same(q, s, q_ref, s_ref):
    assert np.array_equal(q.cpu().numpy(), q_ref)
    assert np.array_equal(s.cpu().view(torch.int16).numpy(), s_ref)


@pytest.mark.parametrize("case", list(golden_cases()), ids=lambda c: c[0])
def test_q8_rows_equals_reference_converter(case):
    _, m, q_ref, s_ref = case
    q, s = convert.q8_rows(m.to(DEV))
    same(q, s, q_ref, s_ref)


@pytest.mark.parametrize("N,K,dtype,scale", [(1, 1, torch.float32, 1.0), (3, 5, torch.float32, 3.0),
                                             (64, 3072, torch.float32, 0.02), (257, 4097, torch.bfloat16, 1.0),
                                             (33, 1024, torch.bfloat16, 1e3), (9, 300, torch.float16, 0.01),
                                             (1500, 256, torch.float32, 1e-9)])
def test_q8_rows_equals_oracle(N, K, dtype, scale):
    g = torch.Generator().manual_seed(N * 7 + K)
    x = (torch.randn(N, K, generator=g) * scale).to(dtype)
    x[0, :] = 0.0
    q, s = convert.q8_rows(x.to(DEV))
    q_ref, s_ref = O.q8_rows(x)
    same(q, s, q_ref.numpy(), s_ref.view(torch.int16).numpy())


@pytest.mark.parametrize("K,ld", [(3072, 3080), (1000, 1001)])
def test_q8_rows_strided_rows(K, ld):
    """Row pitch above K (a column slice of a wider matrix); 4-aligned and ragged."""
    g = torch.Generator().manual_seed(K)
    wide = torch.randn(40, ld, generator=g)
    x = wide[:, :K]
    L = _lib.lib()
    xd = wide.to(DEV)
    q = torch.full((40, ld), 5, dtype=torch.int8, device=DEV)  # output pitch ld too
    s = torch.empty(40, dtype=torch.bfloat16, device=DEV)
    rc = L.hm_q8_rows(xd.data_ptr(), _lib.HM_DT_F32, 40, K, ld, q.data_ptr(), ld, s.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    q_ref, s_ref = O.q8_rows(x)
    same(q[:, :K], s, q_ref.numpy(), s_ref.view(torch.int16).numpy())
    assert bool((q[:, K:] == 5).all())  # nothing written past K


def test_q8_rows_argument_errors():
    L = _lib.lib()
    x = torch.zeros(2, 8, device=DEV)
    q = torch.zeros(2, 8, dtype=torch.int8, device=DEV)
    s = torch.zeros(2, dtype=torch.bfloat16, device=DEV)
    st = torch.cuda.current_stream().cuda_stream
    a = (x.data_ptr(), _lib.HM_DT_F32, 2, 8, 8, q.data_ptr(), 8, s.data_ptr(), st)
    assert L.hm_q8_rows(*a) == 0
    for i, bad in ((1, 7), (2, 0), (3, 0), (4, 7), (6, 7)):
        b = list(a)
        b[i] = bad
        assert L.hm_q8_rows(*b) == _lib.HM_EARG
    assert L.hm_q8_rows(None, *a[1:]) == _lib.HM_EARG


def test_gpu_converter_equals_oracle_conversion(tmp_path):
    fake_official(tmp_path, sharded=True)
    gpu = convert.convert_tensors(tmp_path, device=DEV)
    cpu = convert.convert_tensors(tmp_path, device="cpu", quant=O.q8_rows)
    assert sorted(gpu) == sorted(cpu)
    for k in cpu:
        assert gpu[k].dtype == cpu[k].dtype and gpu[k].device.type == "cpu"
        a, b = gpu[k], cpu[k]
        if a.dtype == torch.bfloat16:
            a, b = a.view(torch.int16), b.view(torch.int16)
        assert torch.equal(a, b), k
